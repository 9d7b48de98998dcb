"""GGUF v3 reader/writer (CPU): format/GgufFile.java behaviour."""
import struct

import numpy as np
import pytest

from auratensor_b200 import gguf, synth
from auratensor_b200.inference import LlamaConfig


def test_parses_minimal_header(tmp_path, kats):
    # format/GgufFileTest.java:22-75
    p = tmp_path / "min.gguf"
    p.write_bytes(bytes.fromhex(kats["gguf_minimal_header_hex"]))
    with gguf.GgufFile.open(str(p)) as g:
        assert g.version == 3
        assert g.tensor_count == 0
        assert g.metadata_kv_count == 1
        assert g.metadata.string_or_default("general.architecture", "") == "llama"


def test_bad_magic_and_version(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(struct.pack("<IIQQ", 0x12345678, 3, 0, 0))
    with pytest.raises(IOError, match="magic"):
        gguf.GgufFile.open(str(p))
    p.write_bytes(struct.pack("<IIQQ", gguf.MAGIC, 2, 0, 0))
    with pytest.raises(IOError, match="version"):
        gguf.GgufFile.open(str(p))


def test_roundtrip_tiny_model(tmp_path):
    shape = synth.TINY
    t = synth.generate_numpy(shape, seed=3)
    p = str(tmp_path / "tiny.gguf")
    synth.write_gguf(shape, t, p)
    with gguf.GgufFile.open(p) as g:
        assert g.data_offset % 32 == 0
        cfg = LlamaConfig.fromGguf(g.metadata)
        assert (cfg.embeddingLength, cfg.blockCount, cfg.headCount, cfg.headCountKv) == (256, 2, 4, 2)
        assert cfg.vocabSize == shape.vocab and cfg.contextLength == shape.ctx
        assert cfg.ropeFrequencyBase == shape.rope_theta
        for name, tt in t.items():
            info = g.find_tensor(name)
            assert info is not None and info.type == tt["type"]
            assert info.num_elements() == int(np.prod(tt["dims"]))
            assert bytes(g.tensor_data(info)) == tt["data"].tobytes()
        assert g.find_tensor("nope") is None
        # the reference's method names are the same calls
        assert g.findTensor("nope") is None
        first = g.tensor_infos[0]
        assert g.findTensor(first.name) is first
        assert bytes(g.tensorData(first)) == bytes(g.tensor_data(first))


def test_config_defaults():
    m = gguf.GgufMetadata({"general.architecture": "llama", "llama.embedding_length": 4096})
    c = LlamaConfig.fromGguf(m)
    assert c.ropeFrequencyBase == 500000.0 and c.vocabSize == 32000 and c.headCountKv == 32
    m = gguf.GgufMetadata({"general.architecture": "llama", "llama.embedding_length": 2048})
    assert LlamaConfig.fromGguf(m).ropeFrequencyBase == 10000.0
    m = gguf.GgufMetadata({"tokenizer.ggml.vocab_size": 777})
    assert LlamaConfig.fromGguf(m).vocabSize == 777


def test_byte_size_rules():
    assert gguf.GgufTensorInfo("a", (64, 32), gguf.Q4_0, 0).byte_size() == 64 * 18
    assert gguf.GgufTensorInfo("a", (64, 32), gguf.Q8_0, 0).byte_size() == 64 * 34
    assert gguf.GgufTensorInfo("a", (256,), 14, 0).byte_size() == 210  # Q6_K super-block
    assert gguf.GgufTensorInfo("a", (10,), gguf.F16, 0).byte_size() == 20


def test_quantizers_roundtrip_through_oracle():
    from oracle import ref
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(32 * 64) * 0.02).astype(np.float32)
    w4 = ref.q4_0_dequant(synth.quantize_q4_0(x), x.size)
    w8 = ref.q8_0_dequant(synth.quantize_q8_0(x), x.size)
    xb = x.reshape(-1, 32)
    amax = np.abs(xb).max(axis=1, keepdims=True)
    # half a step, except a value opposite in sign to the largest one, which clamps at q = 15 (one step)
    assert np.all(np.abs(w4.reshape(-1, 32) - xb) <= amax / 8 + amax * 2e-3)
    assert np.all(np.abs(w8.reshape(-1, 32) - xb) <= amax / 127 * 0.5 + amax * 2e-3)
