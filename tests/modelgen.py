"""Seeded synthetic llama weights for the parity tests, in two views of the same
bytes: the file layout of an import_params.py export (what the library loads)
and the concatenated layout the reference's loader builds (what the oracle
reads, MiniCPM5Weights.cs:139-191)."""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import oracle as orc


@dataclass
class TestConfig:
    hidden: int
    inter: int
    layers: int
    hq: int
    hkv: int
    hd: int
    vocab: int
    quant: str = "int8"
    group: int = 128
    eps: float = 1e-5
    theta: float = 10000.0
    # Gemma3 variants: arch bits (1 qk-norm, 2 sandwich norms, 4 GELU), sliding window / pattern,
    # local RoPE base, softmax scale, embedding scale
    arch: int = 0
    window: int = 0
    pattern: int = 0
    theta_local: float = 0.0
    attn_scale: float = 0.0
    embed_scale: float = 1.0
    # Qwen3.5 full-attention layers: arch bit 8 (q projection with an output gate per head),
    # rotary dims (0 = head_dim)
    rot: int = 0

    def du_kwargs(self):
        from deepunity_b200.llm import LlamaConfig
        return LlamaConfig(self.hidden, self.inter, self.layers, self.hq, self.hkv, self.hd, self.vocab,
                           self.eps, self.theta, group_size=self.group if self.quant == "int4" else 128,
                           arch_flags=self.arch, sliding_window=self.window, sliding_pattern=self.pattern,
                           rope_theta_local=self.theta_local, attn_scale=self.attn_scale,
                           embed_scale=self.embed_scale, rope_rot_dim=self.rot)


SMALL = TestConfig(hidden=256, inter=512, layers=2, hq=4, hkv=2, hd=64, vocab=1024)
MID = TestConfig(hidden=512, inter=1024, layers=2, hq=4, hkv=1, hd=128, vocab=2048)
# BASELINE config 4 (1.1B llama, int8) and a 2-layer slice of config 5 (8B, int4 g128)
C4 = TestConfig(hidden=2048, inter=5632, layers=22, hq=32, hkv=4, hd=64, vocab=32000, quant="int8")
C5_SLICE = TestConfig(hidden=4096, inter=14336, layers=2, hq=32, hkv=8, hd=128, vocab=128256, quant="int4", group=128)


class ModelWeights:
    def __init__(self, cfg: TestConfig, seed: int = 0, std: float = 0.02, gamma_std: float = 0.1):
        self.cfg = cfg
        rng = np.random.default_rng(seed)
        H, I, hd = cfg.hidden, cfg.inter, cfg.hd
        self.files = {}
        self.w_qkv, self.s_qkv, self.w_o, self.s_o, self.w_mlp, self.s_mlp = [], [], [], [], [], []
        self.ln1, self.ln2 = [], []
        self.q_norm, self.k_norm, self.post_attn, self.post_ffn = [], [], [], []
        ext = {"int8": ".int8.bin", "int4": ".int4.bin", "fp16": ".bin"}[cfg.quant]

        def quant(w):
            if cfg.quant == "int8":
                return orc.quantize_int8(w)
            if cfg.quant == "int4":
                return orc.quantize_int4(w, cfg.group)
            return w.astype(np.float16).view(np.uint16), None

        for li in range(cfg.layers):
            qrows = cfg.hq * hd * (2 if cfg.arch & 8 else 1)        # QProjGated: q then gate rows per head
            shapes = {"self_attn_q_proj": (qrows, H), "self_attn_k_proj": (cfg.hkv * hd, H),
                      "self_attn_v_proj": (cfg.hkv * hd, H), "self_attn_o_proj": (H, cfg.hq * hd),
                      "mlp_gate_proj": (I, H), "mlp_up_proj": (I, H), "mlp_down_proj": (H, I)}
            qd = {}
            for name, shp in shapes.items():
                w = (rng.standard_normal(shp, dtype=np.float32) * std).astype(np.float32)
                q, s = quant(w)
                qd[name] = (q, s)
                self.files[f"layer_{li}/{name}{ext}"] = q
                if s is not None:
                    self.files[f"layer_{li}/{name}.scales.bin"] = s
            cat = lambda names, i: np.ascontiguousarray(np.concatenate([qd[n][i].reshape(-1) for n in names]))
            self.w_qkv.append(cat(["self_attn_q_proj", "self_attn_k_proj", "self_attn_v_proj"], 0))
            self.w_o.append(np.ascontiguousarray(qd["self_attn_o_proj"][0].reshape(-1)))
            self.w_mlp.append(cat(["mlp_gate_proj", "mlp_up_proj", "mlp_down_proj"], 0))
            if cfg.quant != "fp16":
                self.s_qkv.append(cat(["self_attn_q_proj", "self_attn_k_proj", "self_attn_v_proj"], 1))
                self.s_o.append(np.ascontiguousarray(qd["self_attn_o_proj"][1].reshape(-1)))
                self.s_mlp.append(cat(["mlp_gate_proj", "mlp_up_proj", "mlp_down_proj"], 1))
            else:
                self.s_qkv.append(None); self.s_o.append(None); self.s_mlp.append(None)
            g1 = (rng.standard_normal(H).astype(np.float32) * gamma_std).astype(np.float16).view(np.uint16)
            g2 = (rng.standard_normal(H).astype(np.float32) * gamma_std).astype(np.float16).view(np.uint16)
            self.ln1.append(g1)
            self.ln2.append(g2)
            self.files[f"layer_{li}/input_layernorm.bin"] = g1
            if cfg.arch & 2:      # sandwich norms: ln2 is the pre-MLP norm under Gemma3's name
                pa = (rng.standard_normal(H).astype(np.float32) * gamma_std).astype(np.float16).view(np.uint16)
                pf = (rng.standard_normal(H).astype(np.float32) * gamma_std).astype(np.float16).view(np.uint16)
                self.post_attn.append(pa)
                self.post_ffn.append(pf)
                self.files[f"layer_{li}/post_attention_layernorm.bin"] = pa
                self.files[f"layer_{li}/pre_feedforward_layernorm.bin"] = g2
                self.files[f"layer_{li}/post_feedforward_layernorm.bin"] = pf
            else:
                self.files[f"layer_{li}/post_attention_layernorm.bin"] = g2
            if cfg.arch & 1:
                qn = (rng.standard_normal(hd).astype(np.float32) * gamma_std).astype(np.float16).view(np.uint16)
                kn = (rng.standard_normal(hd).astype(np.float32) * gamma_std).astype(np.float16).view(np.uint16)
                self.q_norm.append(qn)
                self.k_norm.append(kn)
                self.files[f"layer_{li}/self_attn_q_norm.bin"] = qn
                self.files[f"layer_{li}/self_attn_k_norm.bin"] = kn
        self.final_norm = (rng.standard_normal(H).astype(np.float32) * gamma_std).astype(np.float16).view(np.uint16)
        self.files["norm.bin"] = self.final_norm
        self.embed = (rng.standard_normal((cfg.vocab, H), dtype=np.float32) * std).astype(np.float16).view(np.uint16)
        self.lm_head = (rng.standard_normal((cfg.vocab, H), dtype=np.float32) * std).astype(np.float16).view(np.uint16)
        rows = cfg.vocab // 16
        for k in range(16):
            self.files[f"embed_tokens/part_{k}.bin"] = self.embed[k * rows:(k + 1) * rows]
            self.files[f"lm_head/part_{k}.bin"] = self.lm_head[k * rows:(k + 1) * rows]

    def load_into(self, model):
        for name, arr in self.files.items():
            model.load_tensor(name, arr)
