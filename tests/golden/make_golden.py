"""Generate tests/golden/golden_v21.npz from the reference's OWN CPU code.

The outputs come from oracle/_ref/libptref.so, i.e. runtime/v21/src/pt_v21_host.c compiled from
the reference tree by oracle/Makefile (pt_v21_conv_cpu, pt_v21_convT_cpu and the interpreter's
un_op / bin_op / op_einsum / op_pad / op_slice wired as in ref/v21_graph_trace.txt).  Inputs are
regenerated from seeds at test time, so only seeds, shapes and outputs are stored.

    python tests/golden/make_golden.py        (needs oracle/_ref/libptref.so: make -C oracle)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.join(REPO, "oracle"), os.path.join(REPO, "prime-tts_b200")]

import oracle  # noqa: E402
import pt_b200  # noqa: E402

# conv cases: (seed, B, cin, cout, K, pad, dil, T, epi0, a0, epi1, a1)
CONV_CASES = [
    (10, 1, 32, 16, 3, 1, 1, 40, 0, 0.0, 0, 0.0),
    (11, 2, 40, 72, 7, 3, 1, 33, 1, 0.1, 0, 0.0),
    (12, 1, 64, 64, 11, 25, 5, 70, 1, 0.1, 3, 0.5),
    (13, 1, 4, 1, 63, 0, 1, 200, 0, 0.0, 0, 0.0),
    (14, 3, 16, 8, 5, 2, 3, 9, 2, 0.0, 4, -0.25),
]
# convT cases: (seed, B, cin, cout, K, s, pad, T)
CONVT_CASES = [
    (20, 1, 32, 16, 16, 4, 6, 17),
    (21, 2, 16, 1, 16, 4, 0, 12),
    (22, 1, 4, 4, 4, 4, 0, 30),
    (23, 1, 24, 12, 7, 3, 2, 10),
]


def conv_inputs(seed, B, cin, cout, K, T):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, cin, T)).astype(np.float32)
    x[x < -1.5] = 0.0  # exercise the reference's zero-skip
    W = (0.1 * rng.standard_normal((cout, cin, K))).astype(np.float32)
    b = (0.05 * rng.standard_normal(cout)).astype(np.float32)
    return x, pt_b200.pack_conv(W), b


def convT_inputs(seed, B, cin, cout, K, s, T):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, cin, T)).astype(np.float32)
    W = (0.1 * rng.standard_normal((cin, cout, K))).astype(np.float32)
    b = (0.05 * rng.standard_normal(cout)).astype(np.float32)
    return x, pt_b200.pack_convT(W, s), b


def tail_inputs(seed, Tp):
    rng = np.random.default_rng(seed)
    return (0.5 * rng.standard_normal((72, Tp))).astype(np.float32)


def cfg1_inputs():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 512, 256)).astype(np.float32)
    W = (0.02 * rng.standard_normal((256, 512, 7))).astype(np.float32)
    b = (0.01 * rng.standard_normal(256)).astype(np.float32)
    return x, pt_b200.pack_conv(W), b


def cfg2_inputs():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1, 512, 256)).astype(np.float32)
    W = (0.02 * rng.standard_normal((512, 256, 16))).astype(np.float32)
    b = (0.01 * rng.standard_normal(256)).astype(np.float32)
    return x, pt_b200.pack_convT(W, 4), b


SAMPLE = 4096


def sample_idx(n, seed=99):
    return np.sort(np.random.default_rng(seed).choice(n, size=min(SAMPLE, n), replace=False))


def main():
    ref = oracle.CpuDecoder("reference")
    out = {}
    for i, (seed, B, cin, cout, K, pad, dil, T, e0, a0, e1, a1) in enumerate(CONV_CASES):
        x, wp, b = conv_inputs(seed, B, cin, cout, K, T)
        out[f"conv{i}"] = ref.conv(x, wp, b, cout, K, pad, dil, e0, e1, a0, a1)
    for i, (seed, B, cin, cout, K, s, pad, T) in enumerate(CONVT_CASES):
        x, wp, b = convT_inputs(seed, B, cin, cout, K, s, T)
        out[f"convT{i}"] = ref.convT(x, wp, b, cout, K, s, pad)
    post = tail_inputs(30, 16 * 8 + 1)
    pq = pt_b200.pqmf_synthesis_filter()
    out["tail_T8"] = ref.tail(post, pq)
    out["tail_T3"] = ref.tail(tail_inputs(31, 16 * 3 + 1), pq)   # < 4096 elements: double math
    x, wp, b = cfg1_inputs()
    y1 = ref.conv(x, wp, b, 256, 7, 3, 1, 1, 0, 0.1, 0.0)
    idx = sample_idx(y1.size)
    out["cfg1_idx"], out["cfg1_val"] = idx, y1.ravel()[idx]
    out["cfg1_sum"] = np.array([y1.astype(np.float64).sum(), (y1.astype(np.float64) ** 2).sum()])
    x, wp, b = cfg2_inputs()
    y2 = ref.convT(x, wp, b, 256, 16, 4, 6)
    idx = sample_idx(y2.size)
    out["cfg2_idx"], out["cfg2_val"] = idx, y2.ravel()[idx]
    out["cfg2_sum"] = np.array([y2.astype(np.float64).sum(), (y2.astype(np.float64) ** 2).sum()])
    for T in (8, 13):
        w, z = pt_b200.config3(seed=2, T=T)
        out[f"decode_T{T}"] = ref.decode(w, z)
    np.savez_compressed(os.path.join(HERE, "golden_v21.npz"), **out)
    print("wrote", os.path.join(HERE, "golden_v21.npz"), {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
