"""The reference's own graph interpreter (runtime/v21/src/pt_v21_host.c) decoding through this
library -- the drop-in claim at run time, not only at link time.

oracle/_ref/interp_decode_{cpu,gpu} are built by oracle/Makefile from the reference's sources
(oracle/interp_decode.c #includes the interpreter): both open a container with the interpreter's
own reader (pt_v21_open) and run the decoder's node range (conv_pre .. the PQMF conv) on an
injected latent, the way pt_v21_stream_chunk runs a window (pt_v21_host.c:2859-2900).  The CPU
build executes every conv node with the reference's CPU functions; the GPU build is the
interpreter's CUDA build (-DPT_V21_CUDA) whose PT_CONV / PT_CONVT cases (pt_v21_host.c:3243-3435)
call pt_v21_conv / pt_v21_convT of libpt_b200.so.  The container is written by
tests/ptk_writer.py with every record that node range reads.

* CPU: the interpreter's own decode equals the oracle's decode on the same (fp16-rounded) weights
  bit for bit -- which pins the container format on both sides and the oracle's decoder wiring
  against the reference's graph tables.
* GPU: the interpreter driving this library matches the interpreter on the CPU (SNDR >= 60 dB,
  tests/v21_reference.py:440-447) and the batched decoder built from the same container.
"""
import json
import os
import subprocess

import numpy as np
import pytest

import oracle
import pt_b200
from ptk_writer import decoder_range_tensors, fp16_rounded, write_ptk

REF = os.path.join(os.path.dirname(oracle.LIB_REF))
CPU_BIN = os.path.join(REF, "interp_decode_cpu")
GPU_BIN = os.path.join(REF, "interp_decode_gpu")


def _case(tmp_path, T, seed=2):
    w, z = pt_b200.config3(seed=seed, T=T)
    ptk = str(tmp_path / "dec.ptk")
    write_ptk(ptk, decoder_range_tensors(w))
    zf = str(tmp_path / "z.f32")
    np.ascontiguousarray(z, np.float32).tofile(zf)
    return w, z, ptk, zf


def _run(binary, ptk, zf, T, out, reps=1):
    r = subprocess.run([binary, ptk, zf, str(T), out, str(reps)], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, (r.returncode, r.stderr[-2000:])
    return json.loads(r.stdout.strip().splitlines()[-1]), np.fromfile(out, np.float32)


def test_reference_interpreter_cpu_decode_equals_oracle(tmp_path):
    if not os.path.exists(CPU_BIN):
        pytest.skip("oracle/_ref/interp_decode_cpu not built (needs the reference sources)")
    T = 40
    w, z, ptk, zf = _case(tmp_path, T)
    info, wav = _run(CPU_BIN, ptk, zf, T, str(tmp_path / "wav.f32"))
    assert info["samples"] == 256 * T
    ref = oracle.CpuDecoder("oracle").decode(fp16_rounded(w), z)
    np.testing.assert_array_equal(wav, ref)


@pytest.mark.gpu
def test_reference_interpreter_drives_the_library_on_the_gpu(tmp_path):
    if not (os.path.exists(CPU_BIN) and os.path.exists(GPU_BIN)):
        pytest.skip("oracle/_ref/interp_decode_{cpu,gpu} not built (needs the reference sources)")
    T = 226   # config 3
    w, z, ptk, zf = _case(tmp_path, T)
    cpu_info, cpu_wav = _run(CPU_BIN, ptk, zf, T, str(tmp_path / "cpu.f32"))
    gpu_info, gpu_wav = _run(GPU_BIN, ptk, zf, T, str(tmp_path / "gpu.f32"), reps=3)
    assert gpu_wav.shape == cpu_wav.shape == (256 * T,)
    m = oracle.metrics(gpu_wav, cpu_wav)
    d = pt_b200.Decoder.from_container(ptk)
    try:
        (batched,) = d.decode([z])
    finally:
        d.close()
    mb = oracle.metrics(gpu_wav, batched)
    print(f"\ninterpreter on the GPU vs on the CPU: {m}; vs the batched decoder: {mb}; "
          f"GPU per-op path {gpu_info['s_per_decode'] * 1e3:.1f} ms per decode "
          f"({gpu_info['audio_s_per_s']:.1f} audio-s/s), CPU {cpu_info['s_per_decode']:.2f} s")
    assert np.isfinite(gpu_wav).all()
    assert m["sndr_db"] >= 60.0, m
    assert mb["sndr_db"] >= 60.0, mb
