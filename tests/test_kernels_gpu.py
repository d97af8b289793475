"""Kernel parity on the GPU, through the C ABI, against the CPU oracle.

Tolerances (stated per test): integer work is bit-exact; fp32 outputs are
compared as max|gpu - oracle| / max|oracle| (the norm-wise relative error; the
north-star gate for layer outputs is 1e-3)."""
import ctypes as C

import numpy as np
import pytest
import torch

from deepunity_b200 import _lib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-4     # max-abs error relative to max |y| for one GEMV
ATTN_TOL = 1e-4


@pytest.fixture(scope="module", autouse=True)
def device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    _lib.call("du_init", 0)
    torch.cuda.set_device(0)
    yield


def ptr(t: torch.Tensor):
    return C.c_void_p(t.data_ptr())


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def relerr(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


# ------------------------------------------------------------ quantizers
@pytest.mark.parametrize("rows,cols", [(64, 256), (333, 1024), (4096, 4096)])
def test_device_quantize_int8_bit_exact(rows, cols):
    w = (np.random.default_rng(rows).standard_normal((rows, cols), dtype=np.float32) * 0.02)
    w[0] = 0.0                                   # exercise the 1e-8 floor
    q_ref, s_ref = orc.quantize_int8(w)
    wd = dev(w)
    q = torch.empty((rows, cols), dtype=torch.int8, device="cuda")
    s = torch.empty(rows, dtype=torch.int16, device="cuda")
    _lib.call("du_quantize_int8", ptr(wd), rows, cols, ptr(q), ptr(s), None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), s_ref)


@pytest.mark.parametrize("group", [32, 128])
@pytest.mark.parametrize("rows,cols", [(64, 256), (37, 1024), (4096, 4096)])
def test_device_quantize_int4_bit_exact(rows, cols, group):
    w = (np.random.default_rng(cols).standard_normal((rows, cols), dtype=np.float32) * 0.02)
    w[1, :group] = 0.0                           # 1e-10 floor
    w[2, 5] = 0.5; w[2, 9] = -0.5                # tie on |w|: first index wins
    p_ref, d_ref = orc.quantize_int4(w, group)
    wd = dev(w)
    p = torch.empty((rows, cols // 2), dtype=torch.uint8, device="cuda")
    d = torch.empty((rows, cols // group), dtype=torch.int16, device="cuda")
    _lib.call("du_quantize_int4", ptr(wd), rows, cols, group, ptr(p), ptr(d), None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(p.cpu().numpy(), p_ref)
    np.testing.assert_array_equal(d.cpu().numpy().view(np.uint16), d_ref)


# ---------------------------------------------------- dequantised weights
@pytest.mark.parametrize("quant,group", [("int4", 32), ("int4", 128), ("int8", 0), ("fp16", 0)])
def test_dequant_bit_exact(quant, group):
    """North-star gate: dequantised weight values bit-exact.  du_dequant writes the values
    the tensor-core GEMM's unpack feeds the MMAs (INT4 as its exact fp16 hi + lo pair);
    the oracle is readQ4 / readQ8 * wScale (G3CS:49-101) on the same bytes."""
    rng = np.random.default_rng(7 + group)
    N, K = 300, 4096
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    w[3] = 0.0                                   # quantizer floors
    w[5, :64] *= 1e-3                            # small scales
    w[6, 7] = 0.9                                # one large element per row / group
    if quant == "int8":
        wq, sc = orc.quantize_int8(w)
    elif quant == "int4":
        wq, sc = orc.quantize_int4(w, group)
    else:
        wq, sc = w.astype(np.float16).view(np.uint16), None
    r0, nr = 17, 211
    out = torch.empty((nr, K), dtype=torch.float32, device="cuda")
    wd = dev(wq)
    sd = dev(sc) if sc is not None else None
    qid = {"fp16": _lib.QUANT_FP16, "int8": _lib.QUANT_INT8, "int4": _lib.QUANT_INT4}[quant]
    _lib.call("du_dequant", ptr(out), ptr(wd), ptr(sd) if sd is not None else None, qid, _lib.DTYPE_F16,
              group or 32, r0, nr, K, None)
    torch.cuda.synchronize()
    ref = orc.dequant(wq, sc, quant, N, K, group or 32)[r0:r0 + nr]
    np.testing.assert_array_equal(out.cpu().numpy(), ref)


def test_dequant_real_int8_export_bit_exact():
    """Known-answer data: rows of the reference's shipped int8 export."""
    import os
    ex = np.load(os.path.join(os.path.dirname(__file__), "golden", "int8_export.npz"))
    q, s = ex["q"], ex["s"]
    N, K = q.shape
    out = torch.empty((N, K), dtype=torch.float32, device="cuda")
    qd, sd = dev(q), dev(s)
    _lib.call("du_dequant", ptr(out), ptr(qd), ptr(sd), _lib.QUANT_INT8, _lib.DTYPE_F16, 32, 0, N, K, None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), orc.dequant(q, s, "int8", N, K))


# ------------------------------------------------------------------ GEMM
@pytest.mark.parametrize("quant,group", [("int4", 32), ("int4", 128), ("int8", 0), ("fp16", 0)])
@pytest.mark.parametrize("M,N,K", [(16, 128, 64), (17, 300, 256), (40, 256, 1024), (64, 130, 2048),
                                   (100, 384, 512), (128, 200, 4096), (200, 128, 128)])
def test_gemm_small_shapes(quant, group, M, N, K):
    """The tensor-core GEMM (M >= 16) against the oracle: ragged M and N (partial
    token and row tiles), K from one 64-column block up, every weight format."""
    if quant == "int4" and K % group:
        pytest.skip("K not a multiple of the group")
    rng = np.random.default_rng(M * 7 + N + K)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    x = rng.standard_normal((M, K)).astype(np.float32)
    if quant == "int8":
        wq, sc = orc.quantize_int8(w)
    elif quant == "int4":
        wq, sc = orc.quantize_int4(w, group)
    else:
        wq, sc = w.astype(np.float16).view(np.uint16), None
    ref = orc.gemv(x, wq, sc, quant, N, group or 32)
    y = _gemv(quant, x, wq, sc, N, K, group or 128)
    assert relerr(y, ref) < GEMV_TOL


# ------------------------------------------------------------------ GEMV
def _gemv(quant, x, wq, s, N, K, group=128, scale_f32=False):
    M = x.shape[0]
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    xd, wd = dev(x), dev(wq)
    if quant == "int8":
        sd = dev(s.view(np.float16).astype(np.float32) if scale_f32 else s)
        _lib.call("du_gemv_q8", ptr(y), ptr(xd), _lib.DTYPE_F32, ptr(wd), ptr(sd),
                  _lib.DTYPE_F32 if scale_f32 else _lib.DTYPE_F16, M, N, K, None)
    elif quant == "int4":
        sd = dev(s)
        _lib.call("du_gemv_q4", ptr(y), ptr(xd), _lib.DTYPE_F32, ptr(wd), ptr(sd), group, M, N, K, None)
    else:
        _lib.call("du_gemv_f16", ptr(y), ptr(xd), _lib.DTYPE_F32, ptr(wd), M, N, K, None)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_config1_int8_linear():
    """x [1,1024] ~N(0,1), W [1024,1024] ~N(0,0.02) -> int8 per-row, seed 0,
    with fp16 scales (reference) and fp32 scales (baseline wording)."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((1, 1024)).astype(np.float32)
    w = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    q, s = orc.quantize_int8(w)
    ref = orc.gemv(x, q, s, "int8", 1024)
    for f32 in (False, True):
        y = _gemv("int8", x, q, s, 1024, 1024, scale_f32=f32)
        assert relerr(y, ref) < GEMV_TOL
    # and against the fp32 dequantised matmul of the CPU Dense path
    deq = orc.dequant(q, s, "int8", 1024, 1024)
    dense = orc.dense_linear(x[0], deq)
    assert relerr(y[0], dense) < GEMV_TOL


SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (2560, 2048), (2048, 5632)]


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("quant,group", [("int8", 0), ("int4", 128), ("int4", 32)])
@pytest.mark.parametrize("M", [1, 4])
def test_gemv_matches_oracle(N, K, quant, group, M):
    rng = np.random.default_rng(N + K + M)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02)
    x = rng.standard_normal((M, K), dtype=np.float32)
    if quant == "int8":
        wq, s = orc.quantize_int8(w)
    else:
        wq, s = orc.quantize_int4(w, group)
    ref = orc.gemv(x, wq, s, quant, N, group or 32)
    y = _gemv(quant, x, wq, s, N, K, group or 128)
    assert relerr(y, ref) < GEMV_TOL


@pytest.mark.parametrize("M", [1, 3, 8, 16])
def test_gemv_batch_sizes_and_fp16(M):
    rng = np.random.default_rng(M)
    N, K = 1000, 4096                              # N not a multiple of the CTA row tile
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02)
    x = rng.standard_normal((M, K), dtype=np.float32)
    wh = w.astype(np.float16).view(np.uint16)
    ref = orc.gemv(x, wh, None, "fp16", N)
    assert relerr(_gemv("fp16", x, wh, None, N, K), ref) < GEMV_TOL
    wq, s = orc.quantize_int4(w, 128)
    ref = orc.gemv(x, wq, s, "int4", N, 128)
    assert relerr(_gemv("int4", x, wq, s, N, K), ref) < GEMV_TOL


C2_SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336)]


@pytest.mark.parametrize("N,K", C2_SHAPES)
@pytest.mark.parametrize("quant,group", [("int8", 0), ("int4", 128)])
@pytest.mark.parametrize("M", [16, 64, 512])
def test_config2_batched_tokens(N, K, quant, group, M):
    """BASELINE config 2 at M = 16, 64, 512 with bf16 activations ~N(0,1), W ~N(0,0.02):
    the oracle checks all M tokens on three 256-row windows (first, middle, last)."""
    rng = np.random.default_rng(N + 3 * K + M)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02)
    xb = torch.randn((M, K), generator=torch.Generator().manual_seed(M + K)).to(torch.bfloat16)
    x = xb.float().numpy()
    wq, s = orc.quantize_int8(w) if quant == "int8" else orc.quantize_int4(w, group)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    xd, wd, sd = xb.cuda(), dev(wq), dev(s)
    if quant == "int8":
        _lib.call("du_gemv_q8", ptr(y), ptr(xd), _lib.DTYPE_BF16, ptr(wd), ptr(sd), _lib.DTYPE_F16, M, N, K, None)
    else:
        _lib.call("du_gemv_q4", ptr(y), ptr(xd), _lib.DTYPE_BF16, ptr(wd), ptr(sd), group, M, N, K, None)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    for r0 in (0, N // 2 - 128, N - 256):
        ref = orc.gemv(x, wq, s, quant, 256, group or 32, row_off=r0)
        assert relerr(got[:, r0:r0 + 256], ref) < GEMV_TOL, r0


def test_gemv_real_int8_export_rows():
    """Rows of the reference's shipped int8 export (known-answer data)."""
    import os
    ex = np.load(os.path.join(os.path.dirname(__file__), "golden", "int8_export.npz"))
    q, s = ex["q"], ex["s"]
    N, K = q.shape
    x = np.random.default_rng(5).standard_normal((1, K)).astype(np.float32)
    ref = orc.gemv(x, q, s, "int8", N)
    assert relerr(_gemv("int8", x, q, s, N, K), ref) < GEMV_TOL


def test_gemv_bf16_activations():
    rng = np.random.default_rng(11)
    N, K = 4096, 4096
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02)
    wq, s = orc.quantize_int4(w, 128)
    xb = torch.randn((4, K), generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
    ref = orc.gemv(xb.float().numpy(), wq, s, "int4", N, 128)
    y = torch.empty((4, N), dtype=torch.float32, device="cuda")
    xd, wd, sd = xb.cuda(), dev(wq), dev(s)
    _lib.call("du_gemv_q4", ptr(y), ptr(xd), _lib.DTYPE_BF16, ptr(wd), ptr(sd), 128, 4, N, K, None)
    torch.cuda.synchronize()
    assert relerr(y.cpu().numpy(), ref) < GEMV_TOL


# ------------------------------------------------------------- attention
@pytest.mark.parametrize("hq,hkv,hd", [(32, 8, 128), (32, 4, 64), (8, 8, 128), (16, 8, 64)])
def test_flash_decode_matches_oracle(hq, hkv, hd):
    rng = np.random.default_rng(hq * hd)
    B, cap = 3, 700
    lens = np.array([1, 129, 700], np.int32)
    q = rng.standard_normal((B, hq, hd)).astype(np.float32)
    kc = rng.standard_normal((B, cap, hkv, hd)).astype(np.float16)
    vc = rng.standard_normal((B, cap, hkv, hd)).astype(np.float16)
    scale = 1.0 / np.sqrt(hd)
    out = torch.empty((B, hq, hd), dtype=torch.float32, device="cuda")
    qd, kd, vd, ld = dev(q), dev(kc), dev(vc), dev(lens)
    _lib.call("du_flash_decode", ptr(out), ptr(qd), ptr(kd), ptr(vd), ptr(ld), B, hq, hkv, hd, cap,
              C.c_float(scale), None)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        ref = orc.flash_attention(q[b:b + 1], kc[b].view(np.uint16), vc[b].view(np.uint16), int(lens[b]),
                                  hq, hkv, hd, scale)[0]
        assert relerr(got[b], ref) < ATTN_TOL, b
    # second launch reuses the self-resetting split counters
    _lib.call("du_flash_decode", ptr(out), ptr(qd), ptr(kd), ptr(vd), ptr(ld), B, hq, hkv, hd, cap,
              C.c_float(scale), None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), got)


@pytest.mark.parametrize("ctx,B", [(512, 1), (512, 8), (2048, 8), (2048, 32), (8192, 1), (8192, 8), (8192, 32),
                                   (32768, 1), (32768, 8), (32768, 32)])
def test_flash_decode_baseline_config3(ctx, B):
    """BASELINE config 3 shapes (32 q / 8 kv heads, hd 128) on the model's kernel (the
    thread-block-cluster flash-decode behind du_flash_decode); the oracle checks the first
    and the last sequence."""
    hq, hkv, hd = 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(ctx + B)
    q = torch.randn((B, hq, hd), device="cuda", generator=g)
    kc = torch.randn((B, ctx, hkv, hd), device="cuda", generator=g).half()
    vc = torch.randn((B, ctx, hkv, hd), device="cuda", generator=g).half()
    lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty((B, hq, hd), dtype=torch.float32, device="cuda")
    _lib.call("du_flash_decode", ptr(out), ptr(q), ptr(kc), ptr(vc), ptr(lens), B, hq, hkv, hd, ctx,
              C.c_float(1.0 / np.sqrt(hd)), None)
    torch.cuda.synchronize()
    for b in sorted({0, B - 1}):
        ref = orc.flash_attention(q[b:b + 1].cpu().numpy(), kc[b].cpu().numpy().view(np.uint16),
                                  vc[b].cpu().numpy().view(np.uint16), ctx, hq, hkv, hd, 1.0 / np.sqrt(hd))[0]
        assert relerr(out[b].cpu().numpy(), ref) < ATTN_TOL


def test_rmsnorm_matches_oracle():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 4096)).astype(np.float32)
    g = (rng.standard_normal(4096) * 0.1).astype(np.float16).view(np.uint16)
    ref = orc.rmsnorm(x, g, 1e-5)
    y = torch.empty((5, 4096), dtype=torch.float32, device="cuda")
    xd, gd = dev(x), dev(g)          # keep the device copies alive until the kernel has run
    _lib.call("du_rmsnorm", ptr(y), ptr(xd), ptr(gd), 5, 4096, C.c_float(1e-5), None)
    torch.cuda.synchronize()
    assert relerr(y.cpu().numpy(), ref) < 1e-6


# ----------------------------------------------- Gemma3 attention variants
@pytest.mark.parametrize("hq,hkv,hd,window", [(4, 1, 256, 0), (4, 1, 256, 100), (32, 8, 128, 512), (8, 2, 64, 63)])
def test_flash_decode_window_and_hd256(hq, hkv, hd, window):
    """Sliding-window flash-decode (G3CS:673-686) and head_dim 256 (Gemma3-270M) on the
    cluster kernel, against the oracle's FlashAttention with the same window."""
    rng = np.random.default_rng(hd + window)
    B, cap = 3, 1100
    lens = np.array([40, 700, 1100], np.int32)
    q = rng.standard_normal((B, hq, hd)).astype(np.float32)
    kc = rng.standard_normal((B, cap, hkv, hd)).astype(np.float16)
    vc = rng.standard_normal((B, cap, hkv, hd)).astype(np.float16)
    scale = 1.0 / np.sqrt(hd)
    out = torch.empty((B, hq, hd), dtype=torch.float32, device="cuda")
    args = [dev(a) for a in (q, kc, vc, lens)]
    _lib.call("du_flash_decode_window", ptr(out), *[ptr(a) for a in args], B, hq, hkv, hd, cap, C.c_float(scale),
              window, None)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        ref = orc.flash_attention_window(q[b:b + 1], kc[b].view(np.uint16), vc[b].view(np.uint16), int(lens[b]),
                                         hq, hkv, hd, scale, window)[0]
        assert relerr(got[b], ref) < ATTN_TOL, b


# ------------------------------------------------------------- INT8 KV cache
def _kv_rows(rng, n, hkv, hd):
    """Rows with the reference's edge cases: constant (scale floor), all positive (zp 0),
    all negative (zp clamped to 255, values clipped), half-step ties, a wide range."""
    x = (rng.standard_normal((n, hkv, hd)) * 2).astype(np.float32)
    x[0, 0, :] = 0.25
    x[1 % n, hkv - 1, :] = np.abs(x[1 % n, hkv - 1, :]) + 1.0
    x[2 % n, 0, :] = -np.abs(x[2 % n, 0, :]) - 1.0
    x[3 % n, 0, :] = (np.arange(hd) - hd / 2).astype(np.float32) * (1.0 / 255.0)
    x[4 % n, hkv - 1, ::3] *= 100.0
    return x


@pytest.mark.parametrize("hd", [64, 128])
def test_kv_write_int8_bit_exact(hd):
    """WriteCacheFull's INT8 variant (G3CS:300-380): the cache bytes and the
    (fp16 scale | fp16 zp << 16) words equal the oracle's, bit for bit."""
    rng = np.random.default_rng(hd)
    hkv, n, cap, c0 = 8, 300, 512, 17
    x = _kv_rows(rng, n, hkv, hd)
    q_ref, sz_ref = orc.kv_write_int8(x, hkv, hd)
    cache = torch.zeros((cap, hkv, hd), dtype=torch.uint8, device="cuda")
    sz = torch.zeros((cap, hkv), dtype=torch.int32, device="cuda")
    xd = dev(x)
    _lib.call("du_kv_write_int8", ptr(xd), n, hkv, hd, c0, ptr(cache), ptr(sz), None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache.cpu().numpy()[c0:c0 + n], q_ref)
    np.testing.assert_array_equal(sz.cpu().numpy().view(np.uint32)[c0:c0 + n], sz_ref)
    assert not cache.cpu().numpy()[:c0].any() and not cache.cpu().numpy()[c0 + n:].any()


def _kv8_cache(rng, B, cap, hkv, hd):
    x = (rng.standard_normal((B, cap, hkv, hd))).astype(np.float32)
    q8 = np.empty((B, cap, hkv, hd), np.uint8)
    sz = np.empty((B, cap, hkv), np.uint32)
    for b in range(B):
        q8[b], sz[b] = orc.kv_write_int8(x[b], hkv, hd)
    return q8, sz


@pytest.mark.parametrize("hq,hkv,hd", [(32, 8, 128), (32, 4, 64), (8, 8, 64)])
def test_flash_decode_kv8_matches_oracle(hq, hkv, hd):
    """Flash-decode over the INT8 cache (KV_READ_K / KV_READ_V of KV_INT8) against the
    oracle's FlashAttention on the same bytes, ragged lengths."""
    rng = np.random.default_rng(hq + hd)
    B, cap = 3, 700
    lens = np.array([1, 129, 700], np.int32)
    q = rng.standard_normal((B, hq, hd)).astype(np.float32)
    k8, ksz = _kv8_cache(rng, B, cap, hkv, hd)
    v8, vsz = _kv8_cache(rng, B, cap, hkv, hd)
    scale = 1.0 / np.sqrt(hd)
    out = torch.empty((B, hq, hd), dtype=torch.float32, device="cuda")
    args = [dev(a) for a in (q, k8, ksz.view(np.int32), v8, vsz.view(np.int32), lens)]   # kept alive until the sync
    _lib.call("du_flash_decode_kv8", ptr(out), *[ptr(a) for a in args], B, hq, hkv, hd, cap, C.c_float(scale), None)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(B):
        ref = orc.flash_attention_kv8(q[b:b + 1], k8[b], ksz[b], v8[b], vsz[b], int(lens[b]), hq, hkv, hd, scale)[0]
        assert relerr(got[b], ref) < ATTN_TOL, b


@pytest.mark.parametrize("ctx,B", [(2048, 1), (8192, 8), (32768, 1)])
def test_flash_decode_kv8_config3(ctx, B):
    """BASELINE config 3 shapes over the INT8 cache; the oracle checks the first and last
    sequence."""
    hq, hkv, hd = 32, 8, 128
    rng = np.random.default_rng(ctx + B)
    q = rng.standard_normal((B, hq, hd)).astype(np.float32)
    k8 = rng.integers(0, 256, (B, ctx, hkv, hd), dtype=np.uint8)
    v8 = rng.integers(0, 256, (B, ctx, hkv, hd), dtype=np.uint8)
    def words(n):
        sc = (rng.uniform(0.002, 0.02, n)).astype(np.float16).view(np.uint16).astype(np.uint32)
        zp = rng.integers(0, 256, n).astype(np.float16).view(np.uint16).astype(np.uint32)
        return (sc | (zp << 16)).reshape(B, ctx, hkv)
    ksz, vsz = words(B * ctx * hkv), words(B * ctx * hkv)
    lens = np.full(B, ctx, np.int32)
    out = torch.empty((B, hq, hd), dtype=torch.float32, device="cuda")
    args = [dev(a) for a in (q, k8, ksz.view(np.int32), v8, vsz.view(np.int32), lens)]   # kept alive until the sync
    _lib.call("du_flash_decode_kv8", ptr(out), *[ptr(a) for a in args], B, hq, hkv, hd, ctx,
              C.c_float(1.0 / np.sqrt(hd)), None)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in sorted({0, B - 1}):
        ref = orc.flash_attention_kv8(q[b:b + 1], k8[b], ksz[b], v8[b], vsz[b], ctx, hq, hkv, hd, 1.0 / np.sqrt(hd))[0]
        assert relerr(got[b], ref) < ATTN_TOL, b


# --------------------------------------------------------------- sampler
SAMPLER_SETTINGS = [(0.0, 0, 1.0, 0.0),      # greedy (ArgMax)
                    (1.0, 40, 0.9, 0.0),     # top-k + top-p
                    (0.7, 64, 0.95, 0.05),   # top-k + top-p + min-p
                    (1.3, 1, 1.0, 0.0),      # top-1
                    (1.0, 20, 1.0, 0.2),     # top-k + min-p
                    (1.0, 0, 1.0, 0.0),      # full vocabulary, index-order draw
                    (0.8, 0, 1.0, 0.1)]      # full vocabulary + min-p


def _serial_pick_ok(logits, T, min_p, seed, idx, tol=1e-4):
    """SampleTokenSerial's draw (G3CS:932-1019) on the exact distribution: idx is a valid pick
    for u = runif(seed) if u lies in [cdf(idx - 1), cdf(idx)] up to the fp32 cumulative rounding."""
    u, _ = orc.runif(seed)
    lg = logits.astype(np.float64)
    e = np.exp((lg - lg.max()) / T)
    pr = e / e.sum()
    if min_p > 0:
        pr = np.where(pr >= pr.max() * min_p, pr, 0.0)
    pr = pr / pr.sum()
    c = np.cumsum(pr)
    lo = c[idx - 1] if idx > 0 else 0.0
    return pr[idx] > 0 and lo - tol <= u <= c[idx] + tol


@pytest.mark.parametrize("V", [1000, 32000, 128256])
def test_sampler_matches_oracle(V):
    """SampleToken / SampleTokenSerial (G3CS:932-1132) with runif (G3CS:177-186): identical ids
    for the same logits and seeds on the top-k path and greedy; a pick inside runif's cdf
    interval on the full-vocabulary path."""
    rng = np.random.default_rng(V)
    rows = 8
    logits = (rng.standard_normal((rows, V)) * 3).astype(np.float32)
    logits[1, 100:140] = logits[1].max() + 1.0           # a tie group at the top (tree order decides)
    lg = dev(logits)
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    for (T, k, p, mp) in SAMPLER_SETTINGS:
        for rep in range(3):
            seeds = rng.integers(-2 ** 31, 2 ** 31 - 1, rows, dtype=np.int64).astype(np.int32)
            sd = dev(seeds)
            _lib.call("du_sample", ptr(out), ptr(lg), rows, V, V, C.c_float(T), k, C.c_float(p), C.c_float(mp),
                      ptr(sd), None)
            torch.cuda.synchronize()
            got = out.cpu().numpy().tolist()
            if T > 0 and k <= 0:
                # full-vocabulary path: the reference walks a sequential fp32 cumulative sum over
                # the whole vocabulary (up to ~3e-5 of accumulated rounding at 128K terms, measured
                # on these inputs; the tolerance is 1e-4), so the pick is
                # checked against the exact (float64) distribution: runif(seed) must fall inside the
                # picked token's cdf interval, within that rounding
                for r in range(rows):
                    assert _serial_pick_ok(logits[r], T, mp, int(seeds[r]), got[r]), (T, k, p, mp, rep, r)
                    assert _serial_pick_ok(logits[r], T, mp, int(seeds[r]),
                                           orc.sample(logits[r], T, k, p, mp, int(seeds[r])))
            else:
                ref = [orc.sample(logits[r], T, k, p, mp, int(seeds[r])) for r in range(rows)]
                assert got == ref, (T, k, p, mp, rep)


@pytest.mark.parametrize("V", [1000, 128256])
def test_penalties_and_mark_seen_match_oracle(V):
    """du_apply_penalties (ApplyRepetitionPresencePenalty, Qwen3_5CS.compute:1421-1433)
    bit-exact against the oracle over rows of logits with zero, negative and positive
    values and seen counts of 0..3; du_mark_seen (MarkSampledTokenSeen, :1436-1441)
    adds one per row and skips ids outside the vocabulary."""
    rng = np.random.default_rng(V + 1)
    rows, ld = 4, V + 16
    logits = (rng.standard_normal((rows, V)) * 5).astype(np.float32)
    logits[:, :3] = [0.0, -2.5, 7.0]
    seen = ((rng.random((rows, V)) < 0.05) * rng.integers(1, 4, (rows, V))).astype(np.uint32)
    seen[:, :3] = 1
    seen_pad = np.zeros((rows, ld), np.uint32)
    seen_pad[:, :V] = seen
    lg_pad = np.zeros((rows, ld), np.float32)
    lg_pad[:, :V] = logits
    for presence, repetition in [(0.5, 1.3), (0.0, 1.0), (1.5, 0.8)]:
        lg = dev(lg_pad)
        sn = dev(seen_pad)
        _lib.call("du_apply_penalties", ptr(lg), rows, V, ld, ptr(sn), ld, C.c_float(presence),
                  C.c_float(repetition), None)
        torch.cuda.synchronize()
        got = lg.cpu().numpy()[:, :V]
        ref = orc.apply_penalties(logits, seen, presence, repetition)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (presence, repetition)
        assert np.array_equal(lg.cpu().numpy()[:, V:], lg_pad[:, V:])          # padding untouched
    sn = dev(seen_pad)
    ids = np.array([5, 5, -1, V], np.int32)
    idd = dev(ids)
    for _ in range(2):
        _lib.call("du_mark_seen", ptr(sn), rows, ld, V, ptr(idd), None)
    torch.cuda.synchronize()
    want = seen_pad.copy()
    want[0, 5] += 2
    want[1, 5] += 2
    assert np.array_equal(sn.cpu().numpy(), want)
    rc = _lib.lib().du_apply_penalties(ptr(dev(lg_pad)), rows, V, ld, ptr(sn), ld, C.c_float(0.0), C.c_float(0.0),
                                       None)
    assert rc == _lib.DU_EINVAL                     # repetition_penalty must be > 0


def test_sampler_rejects_unbounded_nucleus():
    lg = torch.zeros((1, 64), device="cuda")
    sd = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().du_sample(ptr(out), ptr(lg), 1, 64, 64, C.c_float(1.0), 0, C.c_float(0.9), C.c_float(0.0), ptr(sd),
                              None)
    assert rc == _lib.DU_EINVAL


_TC_GEMV_CHILD = r"""
import ctypes as C, os, sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from deepunity_b200 import _lib
from oracle import oracle as orc
_lib.call("du_init", 0)
worst = 0.0
for (N, K, G, M) in [(1000, 4096, 128, 1), (4096, 14336, 128, 2), (300, 2048, 32, 1), (2048, 4096, 64, 2)]:
    rng = np.random.default_rng(N + K + G + M)
    w = rng.standard_normal((N, K), dtype=np.float32) * 0.02
    x = rng.standard_normal((M, K)).astype(np.float32)
    wq, sc = orc.quantize_int4(w, G)
    y = torch.empty((M, N), device="cuda")
    xd, wd, sd = torch.from_numpy(x).cuda(), torch.from_numpy(wq).cuda(), torch.from_numpy(sc).cuda()
    P = lambda t: C.c_void_p(t.data_ptr())
    _lib.call("du_gemv_q4", P(y), P(xd), 0, P(wd), P(sd), G, M, N, K, None)
    torch.cuda.synchronize()
    ref = orc.gemv(x, wq, sc, "int4", N, G)
    worst = max(worst, float(np.abs(y.cpu().numpy() - ref).max() / np.abs(ref).max()))
print(worst)
"""


def test_tcgen05_decode_gemv_opt_in():
    """The opt-in tensor-core decode GEMV (tcgen05.mma kind::i8 on nibble x byte-plane operands,
    DU_DECODE_GEMV=tcgen05, read once per process) against the oracle, M = 1 and 2, groups 32-128."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, DU_DECODE_GEMV="tcgen05")
    r = subprocess.run([sys.executable, "-c", _TC_GEMV_CHILD, root], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    assert float(r.stdout.strip().splitlines()[-1]) < GEMV_TOL
