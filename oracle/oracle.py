"""numpy front end for the CPU oracle (liboracle.so, built from du_oracle.c).

TEST INFRASTRUCTURE ONLY: the checker that tests/, ``__graft_entry__.smoke()``
and bench.py's CPU-baseline leg compare the CUDA library against.  The product
package (deepunity_b200) never imports this module.

Each function names the reference code it restates; see du_oracle.c.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

FP16, INT8, INT4 = 0, 1, 2
_QUANT_IDS = {"fp16": FP16, "int8": INT8, "int4": INT4}


def build() -> str:
    """Compile liboracle.so in place (make) if it is missing or stale."""
    src = os.path.join(_HERE, "du_oracle.c")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "-s"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
        P = C.c_void_p
        _lib.orc_f32_to_f16.restype = C.c_uint16
        _lib.orc_f32_to_f16.argtypes = [C.c_float]
        _lib.orc_f16_to_f32.restype = C.c_float
        _lib.orc_f16_to_f32.argtypes = [C.c_uint16]
        _lib.orc_quantize_int8.argtypes = [P, C.c_int64, C.c_int64, P, P]
        _lib.orc_quantize_int4.argtypes = [P, C.c_int64, C.c_int64, C.c_int, P, P]
        _lib.orc_dequant.argtypes = [P, P, C.c_int, C.c_int, C.c_int64, C.c_int64, P]
        _lib.orc_gemv.argtypes = [P, C.c_int, C.c_int, P, P, C.c_int, C.c_int, C.c_int64, C.c_int, P]
        _lib.orc_rmsnorm.argtypes = [P, C.c_int, C.c_int, P, C.c_float, P]
        _lib.orc_rope_table.argtypes = [C.c_int, C.c_int, C.c_float, P, P]
        _lib.orc_rope_apply.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P]
        _lib.orc_rope_apply_partial.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P, P]
        _lib.orc_kv_write.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, P]
        _lib.orc_flash_attention.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                             C.c_float, P]
        _lib.orc_kv_write_int8.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P]
        _lib.orc_flash_attention_window.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                    C.c_float, C.c_int, P]
        _lib.orc_flash_attention_kv8.argtypes = [P, P, P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                 C.c_float, P]
        _lib.orc_argmax.restype = C.c_int
        _lib.orc_argmax.argtypes = [P, C.c_int]
        _lib.orc_forward.restype = C.c_int
        _lib.orc_forward.argtypes = [P, P, C.c_int, C.c_int, P]
        _lib.orc_dense_linear.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P, C.c_int]
        _lib.orc_module_layer_decode.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                                 C.c_float, C.c_float, P, P, P, P, P, P, P, P, P,
                                                 C.c_int, P, C.c_int]
        _lib.orc_max_threads.restype = C.c_int
        _lib.orc_runif.restype = C.c_float
        _lib.orc_runif.argtypes = [C.POINTER(C.c_int32)]
        _lib.orc_sample.restype = C.c_int
        _lib.orc_sample.argtypes = [P, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float, C.c_int32, P]
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


def f32_to_f16_bits(x: float) -> int:
    return int(lib().orc_f32_to_f16(float(x)))


def quantize_int8(w: np.ndarray):
    """import_params.quantize_int8 restated: (int8 [rows, cols], fp16 bits [rows])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.uint16)
    lib().orc_quantize_int8(_p(w), rows, cols, _p(q), _p(s))
    return q, s


def quantize_int4(w: np.ndarray, group: int = 32):
    """import_params.quantize_int4 restated with a group parameter:
    (packed uint8 [rows, cols/2], fp16 bits [rows, cols/group])."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, cols = w.shape
    assert cols % group == 0 and group % 2 == 0
    p = np.empty((rows, cols // 2), np.uint8)
    s = np.empty((rows, cols // group), np.uint16)
    lib().orc_quantize_int4(_p(w), rows, cols, group, _p(p), _p(s))
    return p, s


def dequant(w: np.ndarray, s, quant: str, rows: int, cols: int, group: int = 32) -> np.ndarray:
    out = np.empty((rows, cols), np.float32)
    s_arr = np.ascontiguousarray(s, dtype=np.uint16) if s is not None else None
    lib().orc_dequant(_p(np.ascontiguousarray(w)), _p(s_arr) if s_arr is not None else None,
                      _QUANT_IDS[quant], group, rows, cols, _p(out))
    return out


def gemv(x: np.ndarray, w: np.ndarray, s, quant: str, n_rows: int, group: int = 32,
         row_off: int = 0) -> np.ndarray:
    """Coalesced GEMV/GEMM restatement: y[m, n] for rows [row_off, row_off + n_rows)."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    M, K = x.shape
    y = np.empty((M, n_rows), np.float32)
    s_arr = np.ascontiguousarray(s, dtype=np.uint16) if s is not None else None
    lib().orc_gemv(_p(x), M, K, _p(np.ascontiguousarray(w)), _p(s_arr) if s_arr is not None else None,
                   _QUANT_IDS[quant], group, row_off, n_rows, _p(y))
    return y


def rmsnorm(x: np.ndarray, gamma_m1_bits: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    y = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), x.shape[0], x.shape[1], _p(np.ascontiguousarray(gamma_m1_bits, np.uint16)),
                      eps, _p(y))
    return y


def rope_table(max_seq: int, head_dim: int, theta: float):
    c = np.empty((max_seq, head_dim // 2), np.uint16)
    s = np.empty((max_seq, head_dim // 2), np.uint16)
    lib().orc_rope_table(max_seq, head_dim, theta, _p(c), _p(s))
    return c, s


def rope_apply_partial(buf: np.ndarray, num_heads: int, head_dim: int, rot: int, pos_offset: int, cos_t, sin_t):
    """ApplyRopePartial restated (Qwen3_5CS.compute:367-393) on [seq, heads, hd] in place;
    tables [pos, rot/2] from rope_table(max_seq, rot, theta)."""
    b = np.ascontiguousarray(buf, dtype=np.float32)
    seq = b.size // (num_heads * head_dim)
    lib().orc_rope_apply_partial(_p(b), seq, num_heads, head_dim, rot, pos_offset, _p(cos_t), _p(sin_t))
    return b


def rope_apply(buf: np.ndarray, num_heads: int, head_dim: int, pos_offset: int, cos_t, sin_t):
    b = np.ascontiguousarray(buf, dtype=np.float32).copy()
    seq = b.size // (num_heads * head_dim)
    lib().orc_rope_apply(_p(b), seq, num_heads, head_dim, pos_offset, _p(cos_t), _p(sin_t))
    return b


def flash_attention(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, kv_len: int,
                    hq: int, hkv: int, hd: int, scale: float) -> np.ndarray:
    """FA-1 restatement.  q fp32 [seq_q, hq, hd]; caches fp16 bits [pos, hkv, hd]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    seq_q = q.size // (hq * hd)
    out = np.empty((seq_q, hq, hd), np.float32)
    lib().orc_flash_attention(_p(q), _p(np.ascontiguousarray(k_cache, np.uint16)),
                              _p(np.ascontiguousarray(v_cache, np.uint16)), seq_q, kv_len, hq, hkv, hd,
                              scale, _p(out))
    return out


def flash_attention_window(q: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, kv_len: int,
                           hq: int, hkv: int, hd: int, scale: float, window: int) -> np.ndarray:
    """Sliding-window FA-1 restatement (window <= 0: full attention)."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    seq_q = q.size // (hq * hd)
    out = np.empty((seq_q, hq, hd), np.float32)
    lib().orc_flash_attention_window(_p(q), _p(np.ascontiguousarray(k_cache, np.uint16)),
                                     _p(np.ascontiguousarray(v_cache, np.uint16)), seq_q, kv_len, hq, hkv, hd,
                                     scale, window, _p(out))
    return out


def kv_write_int8(kv_new: np.ndarray, hkv: int, hd: int):
    """WriteCacheFull, INT8 variant, of fp32 rows [seq, hkv, hd] into a fresh cache:
    returns (uint8 [seq, hkv, hd], uint32 (fp16 scale | fp16 zp << 16) [seq, hkv])."""
    x = np.ascontiguousarray(kv_new, dtype=np.float32)
    seq = x.size // (hkv * hd)
    q = np.zeros((seq, hkv, hd), np.uint8)
    sz = np.zeros((seq, hkv), np.uint32)
    lib().orc_kv_write_int8(_p(x), seq, hkv, hd, 0, _p(q), _p(sz))
    return q, sz


def kv8_dequant(q: np.ndarray, sz: np.ndarray) -> np.ndarray:
    """kv_unpack8: (q - zp) * scale, fp16 scale and zp, fp32 result."""
    scale = (sz & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
    zp = (sz >> 16).astype(np.uint16).view(np.float16).astype(np.float32)
    return (q.astype(np.float32) - zp[..., None]) * scale[..., None]


def flash_attention_kv8(q: np.ndarray, k8, ksz, v8, vsz, kv_len: int, hq: int, hkv: int, hd: int,
                        scale: float) -> np.ndarray:
    """FA-1 restatement over an INT8 cache (uint8 [pos, hkv, hd] + scale/zp words [pos, hkv])."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    seq_q = q.size // (hq * hd)
    out = np.empty((seq_q, hq, hd), np.float32)
    lib().orc_flash_attention_kv8(_p(q), _p(np.ascontiguousarray(k8, np.uint8)), _p(np.ascontiguousarray(ksz, np.uint32)),
                                  _p(np.ascontiguousarray(v8, np.uint8)), _p(np.ascontiguousarray(vsz, np.uint32)),
                                  seq_q, kv_len, hq, hkv, hd, scale, _p(out))
    return out


def argmax(logits: np.ndarray) -> int:
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_argmax(_p(lg), lg.size))


def dense_linear(x: np.ndarray, W: np.ndarray, bias=None, threads: int = 0) -> np.ndarray:
    """Dense.Linear restatement on fp32 weights [h_out, h_in]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    W = np.ascontiguousarray(W, dtype=np.float32)
    batched = 1 if x.ndim == 2 else 0
    batch = x.shape[0] if batched else 1
    h_out, h_in = W.shape
    y = np.empty((batch, h_out) if batched else (h_out,), np.float32)
    b = np.ascontiguousarray(bias, np.float32) if bias is not None else None
    lib().orc_dense_linear(_p(x), batch, batched, h_in, h_out, _p(W), _p(b) if b is not None else None,
                           _p(y), threads)
    return y


def runif(seed: int):
    """runif (G3CS:177-186): (u in [0, 1), next seed) from a signed 32-bit seed."""
    sd = C.c_int32(seed)
    u = float(lib().orc_runif(C.byref(sd)))
    return u, int(sd.value)


def sample(logits: np.ndarray, temperature: float, top_k: int, top_p: float, min_p: float, seed: int) -> int:
    """SampleToken / SampleTokenSerial restated (G3CS:932-1132); -1 if the combination is not covered."""
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    scratch = np.empty(lg.size, np.float32)
    return int(lib().orc_sample(_p(lg), lg.size, temperature, top_k, top_p, min_p, seed, _p(scratch)))


def apply_penalties(logits: np.ndarray, seen: np.ndarray, presence: float, repetition: float) -> np.ndarray:
    """ApplyRepetitionPresencePenalty restated (Qwen3_5CS.compute:1421-1433), fp32: for
    every id with a non-zero count, l = l / repetition if l > 0 else l * repetition, then
    l -= presence (once per id).  logits [..., V], seen [..., V] counts; returns a copy."""
    lg = np.array(logits, dtype=np.float32, copy=True)
    m = np.asarray(seen) != 0
    rep, pres = np.float32(repetition), np.float32(presence)
    v = lg[m]
    v = np.where(v > np.float32(0), v / rep, v * rep).astype(np.float32)
    lg[m] = (v - pres).astype(np.float32)
    return lg


def mark_seen(seen: np.ndarray, ids) -> None:
    """MarkSampledTokenSeen restated (Qwen3_5CS.compute:1436-1441) per row: seen[r, ids[r]] += 1."""
    for r, i in enumerate(np.asarray(ids).reshape(-1)):
        if 0 <= int(i) < seen.shape[-1]:
            seen[r, int(i)] += 1


def max_threads() -> int:
    return int(lib().orc_max_threads())


class _OrcModel(C.Structure):
    _fields_ = [("hidden", C.c_int32), ("inter", C.c_int32), ("layers", C.c_int32),
                ("hq", C.c_int32), ("hkv", C.c_int32), ("hd", C.c_int32), ("vocab", C.c_int32),
                ("quant", C.c_int32), ("group", C.c_int32), ("capacity", C.c_int32),
                ("eps", C.c_float), ("theta", C.c_float), ("embed_scale", C.c_float),
                ("w_qkv", C.POINTER(C.c_void_p)), ("s_qkv", C.POINTER(C.c_void_p)),
                ("w_o", C.POINTER(C.c_void_p)), ("s_o", C.POINTER(C.c_void_p)),
                ("w_mlp", C.POINTER(C.c_void_p)), ("s_mlp", C.POINTER(C.c_void_p)),
                ("ln1", C.POINTER(C.c_void_p)), ("ln2", C.POINTER(C.c_void_p)),
                ("final_norm", C.c_void_p), ("embed", C.c_void_p), ("lm_head", C.c_void_p),
                ("rope_cos", C.c_void_p), ("rope_sin", C.c_void_p),
                ("k_cache", C.POINTER(C.c_void_p)), ("v_cache", C.POINTER(C.c_void_p)),
                ("cache_len", C.c_int32), ("kv_quant", C.c_int32),
                ("k_sz", C.POINTER(C.c_void_p)), ("v_sz", C.POINTER(C.c_void_p)),
                ("arch", C.c_int32), ("window", C.c_int32), ("pattern", C.c_int32), ("attn_scale", C.c_float),
                ("rope_cos_local", C.c_void_p), ("rope_sin_local", C.c_void_p),
                ("q_norm", C.POINTER(C.c_void_p)), ("k_norm", C.POINTER(C.c_void_p)),
                ("post_attn_ln", C.POINTER(C.c_void_p)), ("post_ffn_ln", C.POINTER(C.c_void_p)),
                ("rot_dim", C.c_int32), ("rope_cos_partial", C.c_void_p), ("rope_sin_partial", C.c_void_p)]


class OracleModel:
    """One sequence of the reference llama executor (MiniCPM5Model.Forward with
    use_cache = true) over host weights from :class:`tests.modelgen.ModelWeights`."""

    def __init__(self, weights, capacity: int, kv_int8: bool = False):
        cfg = weights.cfg
        self.cfg, self.w = cfg, weights
        L = cfg.layers
        kvt = np.uint8 if kv_int8 else np.uint16
        self.k_cache = [np.zeros((capacity, cfg.hkv, cfg.hd), kvt) for _ in range(L)]
        self.v_cache = [np.zeros((capacity, cfg.hkv, cfg.hd), kvt) for _ in range(L)]
        self.k_sz = [np.zeros((capacity, cfg.hkv), np.uint32) for _ in range(L)]
        self.v_sz = [np.zeros((capacity, cfg.hkv), np.uint32) for _ in range(L)]
        self.rope_cos, self.rope_sin = rope_table(capacity, cfg.hd, cfg.theta)

        def arr(lst):
            a = (C.c_void_p * L)()
            for i, x in enumerate(lst):
                a[i] = _p(x).value if x is not None else None
            return a

        self._keep = []
        m = _OrcModel()
        m.hidden, m.inter, m.layers = cfg.hidden, cfg.inter, L
        m.hq, m.hkv, m.hd, m.vocab = cfg.hq, cfg.hkv, cfg.hd, cfg.vocab
        m.quant, m.group, m.capacity = _QUANT_IDS[cfg.quant], cfg.group, capacity
        m.eps, m.theta, m.embed_scale = cfg.eps, cfg.theta, getattr(cfg, "embed_scale", 1.0)
        for name in ("w_qkv", "s_qkv", "w_o", "s_o", "w_mlp", "s_mlp", "ln1", "ln2"):
            a = arr(getattr(weights, name))
            self._keep.append(a)
            setattr(m, name, C.cast(a, C.POINTER(C.c_void_p)))
        m.final_norm = _p(weights.final_norm).value
        m.embed = _p(weights.embed).value
        m.lm_head = _p(weights.lm_head).value
        m.rope_cos = _p(self.rope_cos).value
        m.rope_sin = _p(self.rope_sin).value
        kc, vc = arr(self.k_cache), arr(self.v_cache)
        ks, vs = arr(self.k_sz), arr(self.v_sz)
        self._keep += [kc, vc, ks, vs]
        m.k_cache = C.cast(kc, C.POINTER(C.c_void_p))
        m.v_cache = C.cast(vc, C.POINTER(C.c_void_p))
        m.k_sz = C.cast(ks, C.POINTER(C.c_void_p))
        m.v_sz = C.cast(vs, C.POINTER(C.c_void_p))
        m.kv_quant = 2 if kv_int8 else 1
        # Gemma3 variants
        m.arch, m.window, m.pattern = getattr(cfg, "arch", 0), getattr(cfg, "window", 0), getattr(cfg, "pattern", 0)
        m.attn_scale = getattr(cfg, "attn_scale", 0.0)
        if m.window > 0:
            tl = getattr(cfg, "theta_local", 0.0) or cfg.theta
            self.rope_cos_local, self.rope_sin_local = rope_table(capacity, cfg.hd, tl)
            m.rope_cos_local, m.rope_sin_local = _p(self.rope_cos_local).value, _p(self.rope_sin_local).value
        # Qwen3.5 full-attention layers: partial RoPE tables [pos, rot/2] over the rotated dims
        rot = getattr(cfg, "rot", 0)
        m.rot_dim = rot
        if 0 < rot < cfg.hd:
            self.rope_cos_partial, self.rope_sin_partial = rope_table(capacity, rot, cfg.theta)
            m.rope_cos_partial = _p(self.rope_cos_partial).value
            m.rope_sin_partial = _p(self.rope_sin_partial).value
        for name in ("q_norm", "k_norm", "post_attn", "post_ffn"):
            lst = getattr(weights, name, [])
            if lst:
                a = arr(lst)
                self._keep.append(a)
                setattr(m, {"post_attn": "post_attn_ln", "post_ffn": "post_ffn_ln"}.get(name, name),
                        C.cast(a, C.POINTER(C.c_void_p)))
        m.cache_len = 0
        self.m = m

    @property
    def cache_len(self) -> int:
        return int(self.m.cache_len)

    def reset(self):
        self.m.cache_len = 0

    def forward(self, ids, last_pos_only: bool = True) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        S = ids.size
        V = self.cfg.vocab
        out = np.empty((V,) if last_pos_only else (S, V), np.float32)
        rc = lib().orc_forward(C.byref(self.m), _p(ids), S, 1 if last_pos_only else 0, _p(out))
        if rc != 0:
            raise RuntimeError("oracle forward: KV cache capacity exceeded")
        return out

    def generate_greedy(self, prompt, steps: int):
        logits = self.forward(prompt)
        toks = []
        for _ in range(steps):
            t = argmax(logits)
            toks.append(t)
            logits = self.forward([t])
        return toks
