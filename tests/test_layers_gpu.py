"""Layer-by-layer parity of the batched decoder, and parity on the whole benchmark workload.

The reference gates its decoder node by node (tests/v21_reference.py:430-447: max|a-b|/max|b| per
graph-node output against a dump, checkpoints written by pt_v21_checkpoints, runtime/v21/src/
pt_v21.h:204-206) and every waveform by SNDR >= 60 dB (:440-447, 505).  Here:

* per op: each of the 40 conv launches of one config-3 decode (T = 226) is recomputed by the CPU
  oracle from the GPU's own inputs to that launch (its checkpointed input, residual and branch-sum
  tensors), so the error is the launch's alone -- TF32 operands, the accumulation order, the fused
  epilogue (bias, LeakyRelu, residual add, branch sum, /3, the reflection-pad row) and the TF32
  rounding of the stored conv inputs.  Gate: max_rel <= 1e-3 (north-star per-op bound).
* accumulated: the same checkpoints against the oracle's own full decode (the reference's style of
  node gate: every upstream difference included).  Gate: 1e-3 as well -- tighter than the
  reference's own per-node bound for its decoder group, 2e-3 (tests/v21_reference.py:497-498).
  The kernels are deterministic (fixed accumulation order, batch-invariant), so these figures are
  the same on every run.
* all 64 config-4 requests (the benchmark workload) against the oracle: SNDR >= 60 dB each.
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np
import pytest

import oracle
import pt_b200

pytestmark = pytest.mark.gpu

PER_OP_GATE = 1e-3
ACCUMULATED_GATE = 1e-3
LR, LR_FINAL = np.float32(0.1), np.float32(0.01)


def leaky(v, a):
    v = np.asarray(v, np.float32)
    return np.where(v >= 0, v, np.float32(a) * v).astype(np.float32)


def per_op_reference(orc, w, z, G):
    """The oracle's output of every conv launch computed from the GPU checkpoints G of its inputs
    (graph wiring: ref/v21_graph_trace.txt nodes 3819-3935)."""
    out = [orc.conv(z[None], w.pre_w, w.pre_b, 512, 7, 3, 1, epi0=1, a0=float(LR))[0]]
    for s in range(2):
        C = 256 if s == 0 else 128
        b = 19 * s
        lvl_in = G[0] if s == 0 else G[19]
        out.append(orc.convT(lvl_in[None], w.ups_w[s], w.ups_b[s], C, 16, 4, 6)[0][:C])
        u = G[1 + b]
        for rb in range(3):
            r, K = 3 * s + rb, pt_b200.RB_KERNELS[rb]
            for j in range(3):
                d = pt_b200.RB_DILATIONS[j]
                x_prev = u if j == 0 else G[3 + b + 6 * rb + 2 * (j - 1)]
                h_in = leaky(x_prev, LR)
                out.append(orc.conv(h_in[None], w.rb_w1[r][j], w.rb_b1[r][j], C, K,
                                    d * (K - 1) // 2, d, epi0=1, a0=float(LR))[0])
                y = orc.conv(G[2 + b + 6 * rb + 2 * j][None], w.rb_w2[r][j], w.rb_b2[r][j], C, K,
                             (K - 1) // 2, 1)[0]
                x = (y + x_prev).astype(np.float32)
                if j < 2:
                    out.append(x)
                elif rb == 0:
                    out.append(x)
                elif rb == 1:
                    out.append((G[7 + b] + x).astype(np.float32))
                else:
                    q = ((G[13 + b] + x) / np.float32(3.0)).astype(np.float32)
                    lv = leaky(q, LR if s == 0 else LR_FINAL)
                    if s == 1:   # reflection pad (1, 0): row -1 mirrors row 1
                        lv = np.concatenate([lv[:, 1:2], lv], axis=1)
                    out.append(lv)
    out.append(orc.conv(G[38][None], w.post_w, w.post_b, 72, 7, 3, 1)[0])
    return out


@pytest.fixture(scope="module")
def cfg3():
    return pt_b200.config3(seed=2, T=226)


@pytest.fixture(scope="module")
def dec(cfg3):
    d = pt_b200.Decoder(cfg3[0], device=0)
    yield d
    d.close()


def test_checkpoint_decode_equals_the_batched_decode(dec, cfg3):
    """The checkpointing decode keeps conv_post's own output and runs the whole tail kernel after
    it; the batched decode computes the windowed iSTFT frames in conv_post's epilogue (the same
    operations in the same order) and runs only the overlap-add and the PQMF after it.  The
    waveforms agree bit for bit (T = 40: the fp32 functions on both paths)."""
    w, z = cfg3
    _, wav = dec.checkpoints(z[:, :40].copy())
    (ref,) = dec.decode([z[:, :40].copy()])
    np.testing.assert_array_equal(wav, ref)


def test_per_layer_parity_config3(dec, cfg3):
    w, z = cfg3
    orc = oracle.CpuDecoder("oracle")
    G, wav = dec.checkpoints(z)
    acc_ref, wav_ref = orc.decode_checkpoints(w, z)
    op_ref = per_op_reference(orc, w, z, G)
    names = oracle.checkpoint_names()
    rows, worst_op, worst_acc = [], (0.0, ""), (0.0, "")
    for i, name in enumerate(names):
        assert G[i].shape == acc_ref[i].shape == op_ref[i].shape, (name, G[i].shape)
        assert np.isfinite(G[i]).all(), name
        m_op = oracle.metrics(G[i], op_ref[i])["max_rel"]
        m_acc = oracle.metrics(G[i], acc_ref[i])["max_rel"]
        rows.append((i, name, m_op, m_acc))
        worst_op = max(worst_op, (m_op, name))
        worst_acc = max(worst_acc, (m_acc, name))
    m_wav = oracle.metrics(wav, wav_ref)
    print("\nlayer | per-op max_rel | accumulated max_rel")
    for i, name, a, b in rows:
        print(f"{i:2d} {name:16s} {a:.3e} {b:.3e}")
    print(f"worst per-op {worst_op}, worst accumulated {worst_acc}, waveform {m_wav}")
    assert worst_op[0] <= PER_OP_GATE, worst_op
    assert worst_acc[0] <= ACCUMULATED_GATE, worst_acc
    assert m_wav["sndr_db"] >= 60.0, m_wav


def test_config4_every_request_matches_oracle(dec, cfg3):
    """All 64 requests of the benchmark workload (config 4, seed 3) decoded in one batch, each
    against the oracle's decode (host threads, one request each)."""
    w = cfg3[0]
    T, zs = pt_b200.config4()
    outs = dec.decode(zs)
    try:
        threads = len(os.sched_getaffinity(0))
    except Exception:
        threads = os.cpu_count() or 1
    orcs = [oracle.CpuDecoder("oracle") for _ in range(threads)]

    def ref(i):
        return orcs[i % threads].decode(w, zs[i])

    order = sorted(range(len(T)), key=lambda i: -T[i])   # longest first: shortest wall time
    with ThreadPoolExecutor(threads) as ex:
        refs = dict(zip(order, ex.map(ref, order)))
    sndr = np.array([oracle.metrics(outs[i], refs[i])["sndr_db"] for i in range(len(T))])
    rel = np.array([oracle.metrics(outs[i], refs[i])["max_rel"] for i in range(len(T))])
    print(f"\nconfig 4, {len(T)} requests ({sum(T)} frames): SNDR min {sndr.min():.2f} "
          f"median {np.median(sndr):.2f} max {sndr.max():.2f} dB; waveform max_rel max "
          f"{rel.max():.2e} (T of the worst: {T[int(np.argmin(sndr))]})")
    assert (sndr >= 60.0).all(), sorted(zip(sndr.tolist(), T))[:4]
