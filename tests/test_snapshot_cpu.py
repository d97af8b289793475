"""The one-file KV snapshot header (du_kv_file_peek) without a GPU: the version-2
prompt-cache layout (Qwen3_5Cache.cs:149-170) written here byte by byte."""
import struct

import pytest

from deepunity_b200 import LlamaForCausalLM


def _header(magic=0x4C4D4B56, version=2, h=0x1122334455667788, fmt=1, tokens=7, layers=3, extra=b"state"):
    return struct.pack("<IiQBiii", magic, version, h, fmt, tokens, layers, len(extra)) + extra


def test_peek_reads_the_header_and_extra(tmp_path):
    p = tmp_path / "a.kv"
    p.write_bytes(_header() + b"\x00" * 10)
    assert LlamaForCausalLM.PeekConversationKV(str(p)) == (0x1122334455667788, 1, 7, 3, b"state")


@pytest.mark.parametrize("bad", [dict(magic=0x4D354B56), dict(version=1), dict(extra=b"x" * 100)])
def test_peek_misses_on_foreign_or_torn_files(tmp_path, bad):
    p = tmp_path / "b.kv"
    data = _header(**bad)
    if "extra" in bad:
        data = data[:40]              # extra length runs past the end of the file
    p.write_bytes(data)
    assert LlamaForCausalLM.PeekConversationKV(str(p)) is None
    assert LlamaForCausalLM.PeekConversationKV(str(tmp_path / "missing.kv")) is None


def test_delete_conversation_kv(tmp_path):
    p = tmp_path / "c.kv"
    p.write_bytes(_header())
    (tmp_path / "c.kv.tmp").write_bytes(b"x")
    LlamaForCausalLM.DeleteConversationKV(str(p))
    assert not p.exists() and not (tmp_path / "c.kv.tmp").exists()
