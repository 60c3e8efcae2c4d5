// ptk.cu -- reader of the reference's weight container (.ptk) for the decoder's tensors.
//
// Layout (tools/export_v21.py:1-40, write_ptk / read_ptk at :232-276; the runtime's reader is the
// C side it mirrors): a 24-byte header <IIIiq> (magic 0x50544B31 "PTK1", version, n_tensor,
// reserved, data_bytes), n_tensor records of 136 bytes <64si4x6qqq> (name, ndim, 6 dims, nelem,
// payload offset), zero padding to a 64-byte boundary, then the payloads (offsets relative to the
// data start).  A payload is fp32 unless the record name ends in "#h" (fp16).  Decoder conv
// weights are stored packed ([cout4/4][K][cin][4], convT phase-major) and fp16 ("#h"); every fp16
// value is exactly representable in TF32, so the tensor cores see the stored weights unchanged.
// Host-only code: no GPU is needed to read a container.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/pt_b200.h"
#include "common.cuh"

using namespace ptb;

namespace {

constexpr uint32_t kMagic = 0x50544B31u;
constexpr size_t kHdr = 24, kRec = 136;

float half_to_float(uint16_t h) {
  const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
  float v;
  if (e == 0) v = std::ldexp((float)m, -24);                      // zero / subnormal
  else if (e == 31) v = m ? NAN : INFINITY;
  else v = std::ldexp((float)(m | 0x400u), (int)e - 25);
  return s ? -v : v;
}

struct Rec {
  std::string name;
  int64_t nelem = 0, off = 0;
};

}  // namespace

struct pt_b200_ptk {
  std::vector<Rec> recs;
  std::vector<std::vector<float>> keep;   // converted payloads handed out by pointer
  pt_b200_dec_weights w{};
};

namespace {

int load_tensor(pt_b200_ptk *k, const std::vector<unsigned char> &raw, size_t data_off,
                const std::string &name, int64_t expect, const float **out) {
  for (const Rec &r : k->recs) {
    if (r.name != name && r.name != name + "#h") continue;
    const bool h = r.name.size() > 2 && r.name.compare(r.name.size() - 2, 2, "#h") == 0;
    const size_t isz = h ? 2 : 4;
    PTB_REQUIRE(r.nelem == expect, "pt_b200: container tensor %s has %lld values, expected %lld",
                r.name.c_str(), (long long)r.nelem, (long long)expect);
    PTB_REQUIRE(r.off >= 0 && data_off + (size_t)r.off + (size_t)r.nelem * isz <= raw.size(),
                "pt_b200: container tensor %s lies outside the file", r.name.c_str());
    std::vector<float> v((size_t)r.nelem);
    const unsigned char *p = raw.data() + data_off + r.off;
    for (int64_t i = 0; i < r.nelem; ++i) {
      if (h) {
        uint16_t x;
        std::memcpy(&x, p + 2 * i, 2);
        v[(size_t)i] = half_to_float(x);
      } else {
        std::memcpy(&v[(size_t)i], p + 4 * i, 4);
      }
    }
    k->keep.push_back(std::move(v));
    *out = k->keep.back().data();
    return 0;
  }
  PTB_REQUIRE(false, "pt_b200: container has no tensor %s", name.c_str());
  return -1;
}

}  // namespace

extern "C" {

pt_b200_ptk *pt_b200_ptk_open(const char *path) {
  if (!path) {
    set_error("pt_b200: NULL container path");
    return nullptr;
  }
  FILE *f = fopen(path, "rb");
  if (!f) {
    set_error("pt_b200: cannot open container %s", path);
    return nullptr;
  }
  std::vector<unsigned char> raw;
  unsigned char buf[1 << 16];
  size_t n;
  while ((n = fread(buf, 1, sizeof(buf), f)) > 0) raw.insert(raw.end(), buf, buf + n);
  fclose(f);
  auto fail = [&](const char *what) {
    set_error("pt_b200: %s: %s", path, what);
    return static_cast<pt_b200_ptk *>(nullptr);
  };
  if (raw.size() < kHdr) return fail("shorter than the container header");
  uint32_t magic, ver, nt;
  std::memcpy(&magic, raw.data(), 4);
  std::memcpy(&ver, raw.data() + 4, 4);
  std::memcpy(&nt, raw.data() + 8, 4);
  if (magic != kMagic) return fail("not a PTK1 container (bad magic)");
  if (raw.size() < kHdr + (size_t)nt * kRec) return fail("truncated record table");
  auto *k = new pt_b200_ptk();
  for (uint32_t i = 0; i < nt; ++i) {
    const unsigned char *r = raw.data() + kHdr + (size_t)i * kRec;
    Rec rec;
    rec.name.assign(reinterpret_cast<const char *>(r), strnlen(reinterpret_cast<const char *>(r), 64));
    std::memcpy(&rec.nelem, r + 64 + 8 + 6 * 8, 8);
    std::memcpy(&rec.off, r + 64 + 8 + 7 * 8, 8);
    k->recs.push_back(rec);
  }
  const size_t data_off = (kHdr + (size_t)nt * kRec + 63) & ~(size_t)63;
  // the decoder's records: packed sizes of the v21_mbistft_16k layers (cout4 = cout here)
  auto conv_n = [](int64_t cout, int64_t K, int64_t cin) { return cout * K * cin; };
  auto convT_n = [](int64_t cin, int64_t cout, int64_t K, int64_t s) {
    return s * cout * ((K + s - 1) / s) * cin;
  };
  static const int kK[3] = {3, 7, 11};
  pt_b200_dec_weights &w = k->w;
  int bad = 0;
  bad |= load_tensor(k, raw, data_off, "dec.conv_pre.wp", conv_n(512, 7, 192), &w.pre_w);
  bad |= load_tensor(k, raw, data_off, "dec.conv_pre.b", 512, &w.pre_b);
  for (int s = 0; s < 2 && !bad; ++s) {
    const int cin = s == 0 ? 512 : 256, c = cin / 2;
    const std::string u = "dec.ups." + std::to_string(s);
    bad |= load_tensor(k, raw, data_off, u + ".wp", convT_n(cin, c, 16, 4), &w.ups_w[s]);
    bad |= load_tensor(k, raw, data_off, u + ".b", c, &w.ups_b[s]);
    for (int rb = 0; rb < 3 && !bad; ++rb) {
      const int r = 3 * s + rb;
      for (int j = 0; j < 3 && !bad; ++j) {
        const std::string b = "dec.resblocks." + std::to_string(r);
        const std::string c1 = b + ".convs1." + std::to_string(j), c2 = b + ".convs2." + std::to_string(j);
        bad |= load_tensor(k, raw, data_off, c1 + ".wp", conv_n(c, kK[rb], c), &w.rb_w1[r][j]);
        bad |= load_tensor(k, raw, data_off, c1 + ".b", c, &w.rb_b1[r][j]);
        bad |= load_tensor(k, raw, data_off, c2 + ".wp", conv_n(c, kK[rb], c), &w.rb_w2[r][j]);
        bad |= load_tensor(k, raw, data_off, c2 + ".b", c, &w.rb_b2[r][j]);
      }
    }
  }
  if (!bad) bad |= load_tensor(k, raw, data_off, "dec.subband_conv_post.wp", conv_n(72, 7, 128), &w.post_w);
  if (!bad) bad |= load_tensor(k, raw, data_off, "dec.subband_conv_post.b", 72, &w.post_b);
  // PQMF synthesis filter: the final Conv 4 -> 1, k63, packed [1][63][4][4] (output channel 0 of
  // the 4-channel block is the real one); the decoder wants the ONNX [1][4][63]
  const float *pq = nullptr;
  if (!bad) bad |= load_tensor(k, raw, data_off, "dec.Conv.wp", 63 * 4 * 4, &pq);
  if (bad) {
    delete k;
    return nullptr;
  }
  std::vector<float> onnx(4 * 63);
  for (int ci = 0; ci < 4; ++ci)
    for (int t = 0; t < 63; ++t) onnx[(size_t)ci * 63 + t] = pq[((size_t)t * 4 + ci) * 4 + 0];
  k->keep.push_back(std::move(onnx));
  w.pqmf = k->keep.back().data();
  return k;
}

int pt_b200_ptk_decoder_weights(const pt_b200_ptk *k, pt_b200_dec_weights *w) {
  PTB_REQUIRE(k && w, "pt_b200: NULL container or weights");
  *w = k->w;
  return 0;
}

void pt_b200_ptk_close(pt_b200_ptk *k) { delete k; }

pt_b200_decoder *pt_b200_decoder_create_from_ptk(int device, const char *path) {
  pt_b200_ptk *k = pt_b200_ptk_open(path);
  if (!k) return nullptr;
  pt_b200_decoder *d = pt_b200_decoder_create(device, &k->w);
  pt_b200_ptk_close(k);
  return d;
}

}  // extern "C"
