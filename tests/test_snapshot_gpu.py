"""Native export-folder loader and KV snapshots on the GPU.

* du_model_load_folder (MiniCPM5Weights' upload pump) gives the same model as
  per-tensor loads of the same files: bit-identical logits.
* "M5KV" v1 folders (M5/MiniCPM5Cache.cs:78-200): header and file sizes as the
  reference writes them; a restored prefix continues like the original (fp16
  subnormals read as zero, as the reference reader does); mismatches are misses.
* One-file version-2 snapshots (fp16 and INT8 caches): a restored prefix
  continues bit-identically; wrong hash / format / torn files and a vetoed
  caller state are misses."""
import os
import struct

import numpy as np
import pytest
import torch

from deepunity_b200 import DUError, KVQuant, LlamaForCausalLM, LLMQuant
from tests.modelgen import SMALL, TestConfig, ModelWeights

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


def _model(cfg, w=None, kv=KVQuant.FP16, cap=128):
    q = {"int8": LLMQuant.INT8, "int4": LLMQuant.INT4, "fp16": LLMQuant.FP16}[cfg.quant]
    m = LlamaForCausalLM(cfg.du_kwargs(), q, kv_quant=kv, max_context_length=cap, seed=None)
    if w is not None:
        w.load_into(m)
    return m


def _export(w, folder):
    for name, arr in w.files.items():
        p = os.path.join(folder, name)
        os.makedirs(os.path.dirname(p), exist_ok=True)
        np.ascontiguousarray(arr).tofile(p)


CFG_HD128 = TestConfig(256, 512, 2, 4, 2, 128, 1024, quant="int4", group=128)


@pytest.mark.parametrize("cfg", [SMALL, CFG_HD128], ids=lambda c: c.quant)
def test_native_folder_loader_matches_tensor_loads(cfg, tmp_path):
    w = ModelWeights(cfg, seed=3)
    _export(w, str(tmp_path))
    a = _model(cfg, w)
    b = _model(cfg)
    assert b.load_params(str(tmp_path)) == len(w.files)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, (1, 12)).astype(np.int32)
    la, _ = a.forward(prompt)
    lb, _ = b.forward(prompt)
    np.testing.assert_array_equal(la, lb)
    (tmp_path / "layer_0" / "bogus.bin").write_bytes(b"\x00" * 4)
    with pytest.raises(DUError):
        b.load_params(str(tmp_path))
    a.Release()
    b.Release()


def _continue(m, tok, n):
    ids, lg = [], []
    for _ in range(n):
        tok = int(m.decode_step([tok])[0])
        ids.append(tok)
        lg.append(m.read_logits(1)[0].copy())
    return ids, np.stack(lg)


def test_m5kv_folder_round_trip(tmp_path):
    cfg = CFG_HD128
    w = ModelWeights(cfg, seed=4)
    a = _model(cfg, w)
    prompt = np.random.default_rng(2).integers(0, cfg.vocab, (1, 40)).astype(np.int32)
    _, nxt = a.forward(prompt)
    folder = str(tmp_path / "m5kv")
    a.SaveCache(folder)
    meta = open(os.path.join(folder, "meta.bin"), "rb").read()
    assert struct.unpack("<6i", meta) == (0x4D354B56, 1, cfg.layers, cfg.hkv, cfg.hd, 40)
    for l in range(cfg.layers):
        for kv in "kv":
            assert os.path.getsize(os.path.join(folder, f"{kv}_cache_layer_{l}.bin")) == 40 * cfg.hkv * cfg.hd * 2
    b = _model(cfg, w)
    assert b.TryLoadCache(folder)
    assert b.cache_len() == 40
    # the restored rows are the saved ones with fp16 subnormals read as zero
    again = str(tmp_path / "again")
    b.SaveCache(again)
    for l in range(cfg.layers):
        for kv in "kv":
            h = np.fromfile(os.path.join(folder, f"{kv}_cache_layer_{l}.bin"), np.uint16)
            h = np.where((h & 0x7C00) == 0, h & 0x8000, h).astype(np.uint16)
            np.testing.assert_array_equal(np.fromfile(os.path.join(again, f"{kv}_cache_layer_{l}.bin"), np.uint16), h)
    ia, la = _continue(a, int(nxt[0]), 16)
    ib, lb = _continue(b, int(nxt[0]), 16)
    assert ia == ib
    assert float(np.max(np.abs(la - lb)) / np.max(np.abs(la))) < 1e-4
    # misses: another model shape, a short file, the INT8 cache
    other = _model(SMALL, ModelWeights(SMALL, seed=4))
    assert not other.TryLoadCache(folder)
    with open(os.path.join(folder, "v_cache_layer_1.bin"), "r+b") as f:
        f.truncate(100)
    c = _model(cfg, w)
    assert not c.TryLoadCache(folder) and c.cache_len() == 0
    k8 = _model(cfg, w, kv=KVQuant.INT8)
    k8.forward(prompt)
    with pytest.raises(DUError):
        k8.SaveCache(str(tmp_path / "k8"))
    assert not k8.TryLoadCache(again)
    for m in (a, b, c, other, k8):
        m.Release()


@pytest.mark.parametrize("kv", [KVQuant.FP16, KVQuant.INT8], ids=["fp16", "int8"])
def test_conversation_snapshot_round_trip(kv, tmp_path):
    cfg = CFG_HD128
    w = ModelWeights(cfg, seed=5)
    a = _model(cfg, w, kv=kv)
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, (1, 30)).astype(np.int32)
    _, nxt = a.forward(prompt)
    path = str(tmp_path / "conv.kv")
    a.SaveConversationKV(path, 0xABCDEF0123456789, extra=b"transcript-3")
    head = LlamaForCausalLM.PeekConversationKV(path)
    assert head == (0xABCDEF0123456789, int(kv), 30, cfg.layers, b"transcript-3")
    b = _model(cfg, w, kv=kv)
    assert not b.TryRestoreConversationKV(path, 0xABCDEF0123456788)          # another context
    assert not b.TryRestoreConversationKV(path, 0xABCDEF0123456789, accept_extra=lambda x: x == b"other")
    assert b.cache_len() == 0
    assert b.TryRestoreConversationKV(path, 0xABCDEF0123456789, accept_extra=lambda x: x == b"transcript-3")
    assert b.cache_len() == 30
    ia, la = _continue(a, int(nxt[0]), 16)
    ib, lb = _continue(b, int(nxt[0]), 16)
    assert ia == ib
    np.testing.assert_array_equal(la, lb)          # the same cache bytes: the same computation
    other_fmt = _model(cfg, w, kv=KVQuant.INT8 if kv == KVQuant.FP16 else KVQuant.FP16)
    assert not other_fmt.TryRestoreConversationKV(path, 0xABCDEF0123456789)
    data = open(path, "rb").read()
    open(path, "wb").write(data[:-1])                                      # torn write
    c = _model(cfg, w, kv=kv)
    assert not c.TryRestoreConversationKV(path, 0xABCDEF0123456789)
    LlamaForCausalLM.DeleteConversationKV(path)
    assert not os.path.exists(path)
    for m in (a, b, c, other_fmt):
        m.Release()
