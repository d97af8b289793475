"""Host-side mirror of DeepUnity's LLM API for the llama decode path.

Mirrors (paths relative to the DeepUnity project root):
  * ``LLMQuant`` / ``KVQuant`` enums        -- LLM/Base/LLM.cs:15-87
  * ``LLM`` (Predict / Generate / Release)  -- LLM/Base/LLM.cs:365-655
  * ``LLMRegistry.Create(id, quant, ...)``  -- LLM/Base/LLMRegistry.cs:61-73
  * ``LlamaForCausalLM`` = MiniCPM5ForCausalLM's role (LLM/MiniCPM5/MiniCPM5.cs) on
    MiniCPM5Model's executor (MiniCPM5Model.cs), backed by libdeepunity_cuda.
Weights come from an ``import_params.py`` export folder (same file names and
formats) or from the library's seeded synthetic initialiser.
"""
from __future__ import annotations

import ctypes as C
import enum
import os
from dataclasses import dataclass, field
from typing import Callable, Iterator, Optional, Sequence

import numpy as np

from . import _lib


class LLMQuant(enum.IntEnum):
    FP16 = _lib.QUANT_FP16
    INT8 = _lib.QUANT_INT8
    INT4 = _lib.QUANT_INT4


class KVQuant(enum.IntEnum):
    FP32 = 0
    FP16 = 1
    INT8 = 2


@dataclass
class LlamaConfig:
    """Architecture constants (the role of MiniCPM5Config.cs:11-37, as data)."""
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads_q: int
    num_heads_kv: int
    head_dim: int
    vocab_size: int
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    tie_embedding: bool = False
    group_size: int = 128
    name: str = "llama"
    # Gemma3 variants on the same kernels (Gemma3Model.cs:315-590); defaults = llama
    arch_flags: int = 0              # _lib.ARCH_QK_NORM | ARCH_SANDWICH | ARCH_GELU
    sliding_window: int = 0          # > 0: sliding-window layers (G3CS:673-686)
    sliding_pattern: int = 0         # every n-th layer (1-based) is full attention
    rope_theta_local: float = 0.0    # RoPE base of the sliding-window layers
    attn_scale: float = 0.0          # softmax scale (0: head_dim^-0.5)
    rope_rot_dim: int = 0            # rotated dims per head (0: head_dim; Qwen3.5 partial RoPE)
    embed_scale: float = 1.0         # embedding multiplier (Gemma3: sqrt(hidden))


# Configurations named by the benchmark (BASELINE configs 4 and 5) and the
# reference's own llama-style model (MiniCPM5Config.cs:11-37).
CONFIGS = {
    "llama-1.1b": LlamaConfig(2048, 5632, 22, 32, 4, 64, 32000, 1e-5, 10000.0, name="llama-1.1b"),
    "llama-8b": LlamaConfig(4096, 14336, 32, 32, 8, 128, 128256, 1e-5, 10000.0, name="llama-8b"),
    "MiniCPM5-1B": LlamaConfig(1536, 4608, 24, 16, 2, 128, 130560, 1e-6, 5_000_000.0, group_size=32,
                               name="MiniCPM5-1B"),
    # Gemma3-270M (LLM/Gemma3/Gemma3Config.cs): 5 sliding-window layers to 1 full, qk-norm,
    # sandwich norms, GELU GLU, sqrt(hidden) embedding scale, tied embedding
    "gemma3-270m": LlamaConfig(640, 2048, 18, 4, 1, 256, 262144, 1e-6, 1_000_000.0, tie_embedding=True,
                               name="gemma3-270m", arch_flags=_lib.ARCH_QK_NORM | _lib.ARCH_SANDWICH | _lib.ARCH_GELU,
                               sliding_window=512, sliding_pattern=6, rope_theta_local=10_000.0,
                               attn_scale=256 ** -0.5, embed_scale=640 ** 0.5),
}


class LLM:
    """Abstract LLM surface (LLM/Base/LLM.cs)."""

    def Predict(self, input_ids, attn_mask=None) -> np.ndarray:
        raise NotImplementedError

    def Generate(self, input_ids, on_token: Optional[Callable[[int], None]] = None,
                 max_new_tokens: int = 64, stop_tokens: Sequence[int] = ()) -> Iterator[int]:
        raise NotImplementedError

    def Release(self):
        raise NotImplementedError


class LlamaForCausalLM(LLM):
    """Llama-style decoder on libdeepunity_cuda (one GPU, or one tensor-parallel rank)."""

    def __init__(self, config: LlamaConfig, quant: LLMQuant = LLMQuant.INT8, kv_quant: KVQuant = KVQuant.FP16,
                 max_context_length: int = 8192, max_batch: int = 1, params_path: Optional[str] = None,
                 seed: Optional[int] = 0, init_std: float = 0.02, device: int = 0,
                 tp_rank: int = 0, tp_size: int = 1, flags: int = 0):
        if kv_quant not in (KVQuant.FP16, KVQuant.INT8):
            raise NotImplementedError("KV cache formats: KVQuant.FP16 and KVQuant.INT8 (the fp32 cache is not built)")
        self.config = config
        self.kv_quant = KVQuant(kv_quant)
        self.quant = LLMQuant(quant)
        self.max_batch = max_batch
        self.capacity = max_context_length
        self.tp_rank, self.tp_size = tp_rank, tp_size
        _lib.call("du_init", device)
        cfg = _lib.ModelConfig()
        cfg.hidden_size, cfg.intermediate_size = config.hidden_size, config.intermediate_size
        cfg.num_layers, cfg.num_heads_q, cfg.num_heads_kv = config.num_layers, config.num_heads_q, config.num_heads_kv
        cfg.head_dim, cfg.vocab_size = config.head_dim, config.vocab_size
        cfg.rms_eps, cfg.rope_theta, cfg.embed_scale = config.rms_eps, config.rope_theta, config.embed_scale
        cfg.arch_flags, cfg.sliding_window, cfg.sliding_pattern = (config.arch_flags, config.sliding_window,
                                                                   config.sliding_pattern)
        cfg.rope_theta_local, cfg.attn_scale = config.rope_theta_local, config.attn_scale
        cfg.rope_rot_dim = config.rope_rot_dim
        cfg.quant, cfg.group_size = int(self.quant), config.group_size
        cfg.kv_capacity, cfg.max_batch = max_context_length, max_batch
        cfg.tp_rank, cfg.tp_size, cfg.tie_embedding = tp_rank, tp_size, int(config.tie_embedding)
        cfg.flags = flags     # FLAG_PERSISTENT: decode steps as one persistent kernel (default: per-stage graph)
        cfg.kv_quant = int(self.kv_quant)   # 1 fp16, 2 INT8 (asymmetric uint8 rows + fp16 scale / zero point)
        h = C.c_void_p()
        _lib.call("du_model_create", C.byref(cfg), C.byref(h))
        self._h = h
        self._busy = False
        if params_path is not None:
            self.load_params(params_path)
        elif seed is not None:
            _lib.call("du_model_init_random", self._h, seed, init_std)

    # ------------------------------------------------------------------ loading
    def load_tensor(self, name: str, data: np.ndarray):
        a = np.ascontiguousarray(data)
        _lib.call("du_model_load_tensor", self._h, name.encode(), a.ctypes.data_as(C.c_void_p), a.nbytes)

    def load_params(self, folder: str) -> int:
        """Loads an import_params.py export folder (MiniCPM5Weights' role) with the native
        loader: every *.bin under `folder`, memory-mapped, placed by its relative name.
        Returns the number of tensors loaded."""
        n = C.c_int(0)
        _lib.call("du_model_load_folder", self._h, os.fsencode(folder), C.byref(n))
        return n.value

    # ---------------------------------------------------------------- KV snapshots
    def SaveCache(self, folder: str, seq: int = 0):
        """MiniCPM5Cache.SaveAsync (M5/MiniCPM5Cache.cs:78-150): the cached prefix of
        sequence `seq` as an "M5KV" v1 folder (fp16 cache only)."""
        _lib.call("du_model_save_cache", self._h, seq, os.fsencode(folder))

    def TryLoadCache(self, folder: str, seq: int = 0) -> bool:
        """MiniCPM5Cache.TryLoadAsync (M5/MiniCPM5Cache.cs:153-200): True when the folder
        matched this model and its rows are now the cached prefix of sequence `seq`."""
        ok = C.c_int(0)
        _lib.call("du_model_load_cache", self._h, seq, os.fsencode(folder), C.byref(ok))
        return bool(ok.value)

    def SaveConversationKV(self, path: str, context_hash: int, extra: bytes = b"", seq: int = 0):
        """LLM.SaveConversationKV (LLMB/LLM.cs:599-607) in the version-2 one-file layout
        (fp16 or INT8 cache), tagged with the caller's context hash and opaque state."""
        buf = C.create_string_buffer(bytes(extra), max(len(extra), 1))
        _lib.call("du_model_save_kv", self._h, seq, os.fsencode(path), C.c_uint64(context_hash & (2 ** 64 - 1)),
                  buf, len(extra))

    @staticmethod
    def PeekConversationKV(path: str):
        """(context_hash, kv_format, tokens, layers, extra) of a saved conversation, or None."""
        valid, h, fmt, tok, nl, xl = C.c_int(0), C.c_uint64(0), C.c_int(0), C.c_int(0), C.c_int(0), C.c_int(0)
        _lib.call("du_kv_file_peek", os.fsencode(path), C.byref(valid), C.byref(h), C.byref(fmt), C.byref(tok),
                  C.byref(nl), None, 0, C.byref(xl))
        if not valid.value:
            return None
        extra = C.create_string_buffer(max(xl.value, 1))
        _lib.call("du_kv_file_peek", os.fsencode(path), C.byref(valid), None, None, None, None, extra, xl.value,
                  C.byref(xl))
        return int(h.value), int(fmt.value), int(tok.value), int(nl.value), extra.raw[:xl.value]

    def TryRestoreConversationKV(self, path: str, context_hash: int, seq: int = 0,
                                 accept_extra: Optional[Callable[[bytes], bool]] = None) -> bool:
        """LLM.TryRestoreConversationKV (LLMB/LLM.cs:622-642): False on any mismatch (hash,
        cache format, layout, sizes) or when `accept_extra` vetoes the saved caller state;
        nothing reaches the device in those cases."""
        head = self.PeekConversationKV(path)
        if head is None or head[0] != (context_hash & (2 ** 64 - 1)):
            return False
        if accept_extra is not None and not accept_extra(head[4]):
            return False
        ok = C.c_int(0)
        _lib.call("du_model_load_kv", self._h, seq, os.fsencode(path), C.c_uint64(context_hash & (2 ** 64 - 1)),
                  C.byref(ok))
        return bool(ok.value)

    @staticmethod
    def DeleteConversationKV(path: str):
        """LLM.DeleteConversationKV (LLMB/LLM.cs:611-616)."""
        for p in (path, path + ".tmp"):
            if os.path.exists(p):
                os.remove(p)

    # ---------------------------------------------------------------- inference
    @property
    def handle(self):
        return self._h

    def init_tp(self, unique_id: bytes, timeout_ms: int = 60000):
        buf = C.create_string_buffer(bytes(unique_id), 128)
        _lib.call("du_tp_init", self._h, buf, timeout_ms)

    def p2p_handle(self) -> bytes:
        """This rank's 64-byte IPC handle for the peer-memory allreduce (after init_tp)."""
        buf = C.create_string_buffer(64)
        _lib.call("du_tp_comm_handle", self._h, buf)
        return buf.raw

    def init_p2p(self, handles):
        """Maps every rank's communication buffer (handles in rank order); decode then reduces
        over NVLink peer memory instead of NCCL.  Every rank must call it before its first decode step."""
        blob = b"".join(bytes(h) for h in handles)
        buf = C.create_string_buffer(blob, len(blob))
        _lib.call("du_tp_comm_open", self._h, buf, len(handles))

    def forward(self, ids, use_cache: bool = True, last_pos_only: bool = True, want_logits: bool = True):
        """MiniCPM5Model.Forward: ids [batch, seq] -> (logits, greedy next ids)."""
        ids = np.ascontiguousarray(np.atleast_2d(np.asarray(ids, dtype=np.int32)))
        B, S = ids.shape
        V = self.config.vocab_size
        logits = None
        if want_logits:
            logits = np.empty((B, V) if last_pos_only else (B, S, V), np.float32)
        nxt = np.empty(B, np.int32)
        _lib.call("du_forward", self._h, ids.ctypes.data_as(C.c_void_p), B, S, int(use_cache), int(last_pos_only),
                  logits.ctypes.data_as(C.c_void_p) if logits is not None else None, nxt.ctypes.data_as(C.c_void_p))
        return logits, nxt

    def Predict(self, input_ids, attn_mask=None) -> np.ndarray:
        """LLM.Predict (MiniCPM5.cs:121-128): logits for every position, stateless."""
        if attn_mask is not None:
            raise NotImplementedError("attention masks are not supported by the decode path")
        ids = np.asarray(input_ids, dtype=np.int32).reshape(1, -1)
        logits, _ = self.forward(ids, use_cache=False, last_pos_only=False)
        return logits[0]

    def decode_step(self, ids) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        out = np.empty_like(ids)
        _lib.call("du_decode_step", self._h, ids.ctypes.data_as(C.c_void_p), ids.size, out.ctypes.data_as(C.c_void_p))
        return out

    def decode_step_sample(self, ids, temperature: float, top_k: int = 0, top_p: float = 1.0, min_p: float = 0.0,
                           seeds=None) -> np.ndarray:
        """One sampled decode step (SampleYielding): temperature / top-k / top-p / min-p with a
        signed 32-bit seed per sequence (random when not given)."""
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        if seeds is None:
            seeds = np.random.default_rng().integers(-2 ** 31, 2 ** 31 - 1, ids.size)
        sd = np.ascontiguousarray(np.asarray(seeds, dtype=np.int64).astype(np.int32).reshape(-1))
        out = np.empty_like(ids)
        _lib.call("du_decode_step_sample", self._h, ids.ctypes.data_as(C.c_void_p), ids.size, C.c_float(temperature),
                  int(top_k), C.c_float(top_p), C.c_float(min_p), sd.ctypes.data_as(C.c_void_p),
                  out.ctypes.data_as(C.c_void_p))
        return out

    def decode_step_sample_ex(self, ids, temperature: float, top_k: int = 0, top_p: float = 1.0, min_p: float = 0.0,
                              presence_penalty: float = 0.0, repetition_penalty: float = 1.0,
                              seeds=None) -> np.ndarray:
        """decode_step_sample with the repetition / presence penalties over the ids this
        entry point has been fed since the last ResetCache (DispatchSampleKernels,
        Qwen3_5Model.cs:1010-1058)."""
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        if seeds is None:
            seeds = np.random.default_rng().integers(-2 ** 31, 2 ** 31 - 1, ids.size)
        sd = np.ascontiguousarray(np.asarray(seeds, dtype=np.int64).astype(np.int32).reshape(-1))
        out = np.empty_like(ids)
        _lib.call("du_decode_step_sample_ex", self._h, ids.ctypes.data_as(C.c_void_p), ids.size,
                  C.c_float(temperature), int(top_k), C.c_float(top_p), C.c_float(min_p), C.c_float(presence_penalty),
                  C.c_float(repetition_penalty), sd.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p))
        return out

    def decode_loop(self, ids, steps: int) -> np.ndarray:
        ids = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        out = np.empty((steps, ids.size), np.int32)
        _lib.call("du_decode_loop", self._h, ids.ctypes.data_as(C.c_void_p), ids.size, steps,
                  out.ctypes.data_as(C.c_void_p))
        return out

    def read_logits(self, batch: int = 1) -> np.ndarray:
        out = np.empty((batch, self.config.vocab_size), np.float32)
        _lib.call("du_read_logits", self._h, out.ctypes.data_as(C.c_void_p), batch)
        return out

    def Generate(self, input_ids, on_token: Optional[Callable[[int], None]] = None,
                 max_new_tokens: int = 64, stop_tokens: Sequence[int] = (), temperature: float = 0.0,
                 top_k: int = 0, top_p: float = 1.0, min_p: float = 0.0, seed: Optional[int] = None,
                 presence_penalty: float = 0.0, repetition_penalty: float = 1.0) -> Iterator[int]:
        """LLM.Generate (MiniCPM5.cs:133-172): prefill the prompt, then one graph-replayed
        decode step per token.  temperature <= 0 is greedy; otherwise every token is drawn by
        the sampler (temperature / top_k / top_p / min_p, SampleYielding M5M:690-705) with
        seeds from `seed`.  The prompt's last token runs as the first decode step so that the
        first new token is sampled on the device too.  presence_penalty / repetition_penalty
        (LLM.cs:438-440; Qwen3_5Model.cs:1010-1058) penalise the ids generated so far from the
        second new token on (the first has nothing to penalise).  Yields token ids (the
        reference yields frames and reports text through a callback)."""
        if self._busy:
            raise RuntimeError("LLM is busy")   # LLM.cs:393-406
        self._busy = True
        try:
            ids = np.asarray(input_ids, np.int32).reshape(-1)
            rng = np.random.default_rng(seed)
            penalized = presence_penalty != 0.0 or repetition_penalty != 1.0
            if temperature > 0.0:
                if ids.size > 1:
                    self.forward(ids[None, :-1], use_cache=True, want_logits=False)
                step = lambda t: int(self.decode_step_sample([t], temperature, top_k, top_p, min_p,
                                                             [int(rng.integers(-2 ** 31, 2 ** 31 - 1))])[0])
                tok = step(int(ids[-1]))
            else:
                _, nxt = self.forward(ids[None, :], use_cache=True, want_logits=False)
                tok = int(nxt[0])
                step = lambda t: int(self.decode_step([t])[0])
            if penalized:     # each later step's input (the previous pick) is counted as seen
                step = lambda t: int(self.decode_step_sample_ex(
                    [t], temperature, top_k, top_p, min_p, presence_penalty, repetition_penalty,
                    [int(rng.integers(-2 ** 31, 2 ** 31 - 1))])[0])
            for _ in range(max_new_tokens):
                if on_token:
                    on_token(tok)
                yield tok
                if tok in stop_tokens:
                    break
                tok = step(tok)
        finally:
            self._busy = False

    def ResetCache(self):
        _lib.call("du_reset_cache", self._h)

    def cache_len(self, seq: int = 0) -> int:
        v = C.c_int()
        _lib.call("du_cache_len", self._h, seq, C.byref(v))
        return v.value

    def weight_bytes(self) -> int:
        v = C.c_uint64()
        _lib.call("du_model_weight_bytes", self._h, C.byref(v))
        return v.value

    def stream(self) -> int:
        v = C.c_void_p()
        _lib.call("du_model_stream", self._h, C.byref(v))
        return v.value or 0

    def Release(self):
        """Idempotent (LLM.cs:654-655)."""
        if getattr(self, "_h", None) is not None and self._h.value:
            _lib.call("du_model_destroy", self._h)
            self._h = C.c_void_p()

    def __del__(self):
        try:
            self.Release()
        except Exception:
            pass


class LLMRegistry:
    """LLMRegistry.Create (LLMRegistry.cs:61-73) over the configurations above."""

    @staticmethod
    def Create(model_id: str, quant: LLMQuant = LLMQuant.INT8, kv_quant: KVQuant = KVQuant.FP16,
               max_context_length: int = 8192, **kw) -> LlamaForCausalLM:
        if model_id not in CONFIGS:
            raise KeyError(f"unknown model id {model_id!r}; known: {sorted(CONFIGS)}")
        return LlamaForCausalLM(CONFIGS[model_id], quant, kv_quant, max_context_length, **kw)
