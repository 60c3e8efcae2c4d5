"""Request-parallel sharding across ranks (CPU, world_size 2 over gloo).

The decoder path shards into independent requests with no collective on the data path; the only
cross-rank traffic is bench.py's timing barrier and max-over-ranks reduction.  Here two gloo ranks
each take their LPT shard of the config-4 workload, decode it with the CPU oracle (tiny latents so
the test stays fast) and the gathered results must equal the single-rank decode.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [REPO, os.path.join(REPO, "prime-tts_b200"), os.path.join(REPO, "oracle")]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_lpt_shards_balance_and_cover():
    import bench
    T, _ = __import__("pt_b200").config4(seed=3, n=128)
    for n in (1, 2, 4, 8):
        shards = bench.lpt_shards(T, n)
        assert sorted(i for s in shards for i in s) == list(range(len(T)))
        loads = [sum(T[i] for i in s) for s in shards]
        # LPT guarantee: max load <= mean + max job
        assert max(loads) <= sum(T) / n + max(T)


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import bench
    import oracle
    import pt_b200
    rng = np.random.default_rng(9)
    T = [int(t) for t in rng.integers(2, 6, size=6)]
    zs = [rng.standard_normal((192, t)).astype(np.float32) for t in T]
    w = pt_b200.make_decoder_weights(np.random.default_rng(2))
    mine = bench.lpt_shards(T, world)[rank]
    cpu = oracle.CpuDecoder("oracle")
    res = {i: cpu.decode(w, zs[i]) for i in mine}
    gathered = [None] * world
    dist.all_gather_object(gathered, res)
    if rank == 0:
        merged = {}
        for g in gathered:
            merged.update(g)
        out.put({i: merged[i].tolist() for i in sorted(merged)})
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_match_single_rank():
    if not os.path.exists(os.path.join(REPO, "oracle", "liboracle.so")):
        pytest.skip("oracle not built")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    import oracle
    import pt_b200
    rng = np.random.default_rng(9)
    T = [int(t) for t in rng.integers(2, 6, size=6)]
    zs = [rng.standard_normal((192, t)).astype(np.float32) for t in T]
    w = pt_b200.make_decoder_weights(np.random.default_rng(2))
    cpu = oracle.CpuDecoder("oracle")
    assert sorted(got) == list(range(len(T)))
    for i in range(len(T)):
        assert np.array_equal(np.asarray(got[i], np.float32), cpu.decode(w, zs[i]))


def _gpu_count():
    try:
        import torch
        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


@pytest.mark.gpu
@pytest.mark.skipif(_gpu_count() < 2, reason="needs two GPUs")
def test_interpreter_contexts_on_two_devices_agree():
    """Request-parallel interpreter use: a context bound to device 1 (pt_v21_cuda_init_dev) runs
    the same convs as one on device 0 -- a small-N conv (the window kernel) and a 256-channel
    conv (the channels-on-M kernel), each kernel's shared-memory opt-in made on each device --
    and returns the same bits."""
    import pt_b200
    rng = np.random.default_rng(31)
    x = rng.standard_normal((1, 128, 300)).astype(np.float32)
    cases = [(48, 7, 3), (256, 3, 1)]
    outs = {}
    for dev in (0, 1):
        with pt_b200.Context(device=dev) as ctx:
            res = []
            for cout, K, pad in cases:
                W = (0.02 * rng.standard_normal((cout, 128, K))).astype(np.float32) if dev == 0 \
                    else outs[("w", cout)]
                outs[("w", cout)] = W
                b = np.zeros(cout, np.float32)
                res.append(ctx.conv(x, pt_b200.pack_conv(W), b, cout=cout, K=K, pad=pad))
            outs[dev] = res
    for a, b in zip(outs[0], outs[1]):
        np.testing.assert_array_equal(a, b)
