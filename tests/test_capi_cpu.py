"""CPU-side checks of the C ABI: the library loads, exports every symbol the
header declares, and rejects bad arguments with a status (no GPU needed)."""
import ctypes as C
import os
import re

import pytest

from deepunity_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "deepunity_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"DU_API\s+[\w\s\*]+?\b(du_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), f"{n} declared in deepunity_cuda.h but not exported"
    # and the Python binding covers the same set
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_version_and_error_string():
    assert b"sm_100a" in _lib.lib().du_version()
    assert isinstance(_lib.last_error(), str)


def _cfg(**kw):
    c = _lib.ModelConfig()
    c.hidden_size, c.intermediate_size, c.num_layers = 256, 512, 2
    c.num_heads_q, c.num_heads_kv, c.head_dim, c.vocab_size = 4, 2, 64, 1024
    c.rms_eps, c.rope_theta, c.embed_scale = 1e-5, 10000.0, 1.0
    c.quant, c.group_size, c.kv_capacity, c.max_batch, c.tp_rank, c.tp_size = 1, 128, 64, 1, 0, 1
    for k, v in kw.items():
        setattr(c, k, v)
    return c


@pytest.mark.parametrize("bad", [dict(num_heads_q=3), dict(head_dim=96), dict(quant=7),
                                 dict(quant=2, group_size=48), dict(tp_size=2, tp_rank=2),
                                 dict(tp_size=3), dict(max_batch=0), dict(hidden_size=250),
                                 # Qwen3.5 attention gate without qk-norm, or over two ranks
                                 dict(arch_flags=8), dict(arch_flags=9, tp_size=2, tp_rank=0),
                                 # partial RoPE: half not a power-of-two multiple of hd/32, odd,
                                 # above head_dim, or without qk-norm
                                 dict(arch_flags=1, rope_rot_dim=48), dict(arch_flags=1, rope_rot_dim=33),
                                 dict(arch_flags=1, rope_rot_dim=128), dict(rope_rot_dim=32)])
def test_model_create_rejects_bad_config(bad):
    h = C.c_void_p()
    rc = _lib.lib().du_model_create(C.byref(_cfg(**bad)), C.byref(h))
    assert rc == _lib.DU_EINVAL, _lib.last_error()
    assert h.value is None


def test_penalty_entry_points_validate_before_touching_the_device():
    """du_apply_penalties / du_mark_seen / du_decode_step_sample_ex reject bad arguments
    with a status (no GPU needed)."""
    L = _lib.lib()
    p = C.c_void_p(16)
    assert L.du_apply_penalties(None, 1, 8, 8, p, 8, C.c_float(0.0), C.c_float(1.0), None) == _lib.DU_EINVAL
    assert L.du_apply_penalties(p, 1, 8, 4, p, 8, C.c_float(0.0), C.c_float(1.0), None) == _lib.DU_EINVAL  # ldl < vocab
    assert L.du_apply_penalties(p, 1, 8, 8, p, 8, C.c_float(0.0), C.c_float(-1.0), None) == _lib.DU_EINVAL
    assert L.du_mark_seen(p, 1, 4, 8, p, None) == _lib.DU_EINVAL                                      # ld < vocab
    assert L.du_mark_seen(None, 1, 8, 8, p, None) == _lib.DU_EINVAL
    assert L.du_decode_step_sample_ex(None, None, 1, C.c_float(0.0), 0, C.c_float(1.0), C.c_float(0.0),
                                      C.c_float(0.0), C.c_float(1.0), None, None) != 0


def test_kernel_entry_points_validate_before_touching_the_device():
    L = _lib.lib()
    assert L.du_gemv_q4(None, None, 0, None, None, 128, 1, 1, 128, None) == _lib.DU_EINVAL
    assert L.du_gemv_q8(C.c_void_p(16), C.c_void_p(16), 0, C.c_void_p(16), C.c_void_p(16), 9, 1, 1, 16,
                        None) == _lib.DU_EINVAL
    assert L.du_flash_decode(None, None, None, None, None, 1, 32, 8, 128, 64, 0.1, None) == _lib.DU_EINVAL
    assert L.du_forward(None, None, 1, 1, 1, 1, None, None) == _lib.DU_EINVAL
    assert L.du_model_destroy(None) == _lib.DU_OK


def test_init_without_gpu_reports_an_error():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    rc = _lib.lib().du_init(0)
    assert rc != _lib.DU_OK
    assert _lib.last_error()


def test_timing_build_compiles_and_stays_out_of_the_library():
    """The GEMV timing build (gemv.cu with DU_GEMV_STAMPS: per-CTA phase stamps
    for bench.py --gemv-phases) still compiles for sm_100a, and the library proper
    exports none of its symbols (the hook compiles to nothing there)."""
    import shutil
    import subprocess
    import tempfile
    from deepunity_b200 import build as B
    try:
        nvcc = B.nvcc()
    except RuntimeError:
        pytest.skip("nvcc not available")
    assert not hasattr(_lib.lib(), "du_gemv_stamps_read")
    with tempfile.TemporaryDirectory() as d:
        obj = os.path.join(d, "gemv_stamps.o")
        r = subprocess.run([nvcc, "-c", os.path.join(B.CSRC, "gemv.cu"), "-o", obj] + B.ARCH +
                           ["-O1", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-DDU_GEMV_STAMPS"],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stdout + r.stderr
        nm = shutil.which("nm")
        if nm:
            syms = subprocess.run([nm, obj], capture_output=True, text=True).stdout
            assert "du_gemv_stamps_read" in syms and "du_gemv_stamps_reset" in syms
