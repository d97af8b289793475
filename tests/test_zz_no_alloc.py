"""du_flash_decode_noalloc: the flash-decode entry point for callers that must
not allocate device memory (for example a game engine plugin on its render
thread, where the engine owns the GPU memory and cudaMalloc / cudaFree can
stall the whole device).  Its scratch is a fixed device array inside the
library, shared by every call.

The test calls both entry points through the C ABI on the same inputs, twice
in a row (the second call finds the array holding the first call's contents),
and requires the same outputs within the flash-decode tolerance of the other
GPU tests.  The file name sorts last so a run that stops at the first failure
has already run every other test."""
import ctypes as C

import numpy as np
import pytest
import torch

from deepunity_b200 import _lib

pytestmark = pytest.mark.gpu
ATTN_TOL = 1e-4   # max |a - b| / max |b|, as in test_kernels_gpu.py


def _p(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("hq,hkv,hd,batch,cap", [(32, 8, 128, 1, 4096), (32, 4, 64, 3, 700)])
def test_noalloc_matches_allocating_entry_point(hq, hkv, hd, batch, cap):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.call("du_init", 0)
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(hq + hd + batch)
    q = torch.randn((batch, hq, hd), device="cuda", generator=g)
    kc = torch.randn((batch, cap, hkv, hd), device="cuda", generator=g).half()
    vc = torch.randn((batch, cap, hkv, hd), device="cuda", generator=g).half()
    lens = torch.tensor([cap - 17 * b for b in range(batch)], dtype=torch.int32, device="cuda")
    scale = C.c_float(hd ** -0.5)
    ref = torch.empty((batch, hq, hd), device="cuda")
    _lib.call("du_flash_decode", _p(ref), _p(q), _p(kc), _p(vc), _p(lens), batch, hq, hkv, hd, cap, scale, None)
    for _ in range(2):
        out = torch.full((batch, hq, hd), float("nan"), device="cuda")
        _lib.call("du_flash_decode_noalloc", _p(out), _p(q), _p(kc), _p(vc), _p(lens), batch, hq, hkv, hd, cap,
                  scale, None)
        torch.cuda.synchronize()
        a, b = out.cpu().numpy(), ref.cpu().numpy()
        assert np.isfinite(a).all()
        assert float(np.max(np.abs(a - b)) / np.max(np.abs(b))) < ATTN_TOL
    # and directly against the CPU oracle's restatement of FlashAttention (G3CS:643-753)
    from oracle import oracle as orc
    qn, kn, vn = q.cpu().numpy(), kc.cpu().numpy().view(np.uint16), vc.cpu().numpy().view(np.uint16)
    for s in sorted({0, batch - 1}):
        o = orc.flash_attention(qn[s:s + 1], kn[s], vn[s], int(lens[s].item()), hq, hkv, hd, hd ** -0.5)[0]
        assert float(np.max(np.abs(a[s] - o)) / np.max(np.abs(o))) < ATTN_TOL, s


def test_noalloc_rejects_sizes_beyond_its_fixed_scratch():
    """Sizes beyond the fixed array, and head shapes the kernel does not serve,
    return DU_EINVAL before anything is enqueued."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.call("du_init", 0)
    x = torch.zeros(16, device="cuda")
    # batch * num_heads_kv above the 8192 counters
    rc = _lib.lib().du_flash_decode_noalloc(_p(x), _p(x), _p(x), _p(x), _p(x), 1025, 64, 8, 128, 64,
                                            C.c_float(0.1), None)
    assert rc == _lib.DU_EINVAL and "8192" in _lib.last_error()
    # one split of partials above the 1048576-float array
    rc = _lib.lib().du_flash_decode_noalloc(_p(x), _p(x), _p(x), _p(x), _p(x), 300, 32, 8, 128, 64,
                                            C.c_float(0.1), None)
    assert rc == _lib.DU_EINVAL and "1048576" in _lib.last_error()
    # head_dim the kernel does not serve (would size the scratch from a bad value)
    rc = _lib.lib().du_flash_decode_noalloc(_p(x), _p(x), _p(x), _p(x), _p(x), 1, 32, 8, -2, 64,
                                            C.c_float(0.1), None)
    assert rc == _lib.DU_EINVAL and "head_dim" in _lib.last_error()
    # GQA group above 8
    rc = _lib.lib().du_flash_decode_noalloc(_p(x), _p(x), _p(x), _p(x), _p(x), 1, 32, 2, 128, 64,
                                            C.c_float(0.1), None)
    assert rc == _lib.DU_EINVAL and "at most 8" in _lib.last_error()
