"""The GGUF reader (wl_gguf_*, the reference's GgufFile::parse,
src/gguf/reader.rs:120-415) and the model-config reader
(ModelConfig::from_gguf_metadata, src/model/config.rs:61-260), on CPU: round
trips of synthetic files, and the reference's own reader tests
(reader.rs:819-933) restated with the same inputs and message checks."""
import struct

import numpy as np
import pytest

from project_willamette_b200 import WillametteError, gguf, synth
from project_willamette_b200._abi import WLStatus


def _err(data):
    with pytest.raises(WillametteError) as e:
        gguf.GgufFile(data)
    return e.value


def _header(n_tensors, n_kv):
    return struct.pack("<IIQQ", 0x46554747, 3, n_tensors, n_kv)


def _build(infos, tensor_data: bytes) -> bytes:
    """reader.rs build_gguf: tensor infos (name, shape, type, offset), no
    metadata, data section at the next 32-byte boundary."""
    b = _header(len(infos), 0)
    for name, shape, t, off in infos:
        b += gguf._s(name) + struct.pack("<I", len(shape)) + \
            b"".join(struct.pack("<Q", d) for d in shape) + struct.pack("<IQ", t, off)
    b += bytes((-len(b)) % 32)
    return b + tensor_data


def test_bitnet_round_trip():
    m = synth.bitnet_model(np.random.default_rng(2), n_layers=2, n_embd=256, n_heads=2,
                           n_kv_heads=1, n_ff=512, vocab=300, max_seq=32)
    f = gguf.GgufFile(gguf.bitnet_gguf(m))
    assert f.version == 3 and f.alignment == 32 and len(f) == 2 + 2 * 11
    assert f.str("general.architecture") == "bitnet-b1.58"
    assert f.u64("bitnet-b1.58.block_count") == 2
    cfg, variant = f.model_config()
    assert variant == 0
    for k in ("n_layers", "n_embd", "n_heads", "n_kv_heads", "head_dim", "n_ff", "vocab",
              "n_rot", "max_seq"):
        assert cfg[k] == m["config"][k], k
    assert np.float32(cfg["eps"]) == np.float32(m["config"]["eps"])
    emb = f.tensor("token_embd.weight")
    assert emb["type"] == gguf.GGML_Q6_K and emb["shape"] == (256, 300)
    assert np.array_equal(emb["data"], m["token_embd"])
    for l in range(2):
        for k, role in enumerate(["attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate",
                                  "ffn_up", "ffn_down"]):
            t = f.tensor(f"blk.{l}.{role}.weight")
            assert t["type"] == gguf.GGML_I2_S
            assert np.array_equal(t["data"], m["w"][l * 7 + k])
            sb = t["scale_block"]
            assert sb.size == 32 and not sb[4:].any()
            assert np.frombuffer(sb[:4].tobytes(), np.float32)[0] == np.float32(m["w_scale"][l * 7 + k])
    with pytest.raises(WillametteError) as e:
        f.tensor("blk.2.attn_q.weight")
    assert e.value.status == WLStatus.MISSING_METADATA


def test_llama_round_trip_and_config():
    m = synth.llama_q8_model(np.random.default_rng(3), n_layers=1, n_embd=128, n_heads=2,
                             n_kv_heads=1, n_ff=256, vocab=100, max_seq=16)
    f = gguf.GgufFile(gguf.llama_gguf(m))
    cfg, variant = f.model_config()
    assert variant == 1 and cfg["vocab"] == 100 and cfg["head_dim"] == 64
    assert cfg["n_rot"] == 64 and cfg["freq_base"] == 10000.0
    assert f.array_len("tokenizer.ggml.tokens") == 100
    t = f.tensor("blk.0.ffn_down.weight")
    assert t["type"] == gguf.GGML_Q8_0 and t["shape"] == (256, 128)
    assert np.array_equal(t["data"], m["w"][6]) and "scale_block" not in t


def test_i2s_byte_lengths_of_the_real_shapes():
    # tensor.rs:476-489: packed bytes of the 2B model's I2_S shapes
    cases = [((6912, 2560), 4_423_680), ((2560, 6912), 4_423_680), ((2560, 2560), 1_638_400),
             ((2560, 640), 409_600)]
    tensors = [(f"t{i}", s, gguf.GGML_I2_S, bytes(n), 0.5) for i, (s, n) in enumerate(cases)]
    f = gguf.GgufFile(gguf.write_gguf({}, tensors))
    for i, (_, n) in enumerate(cases):
        assert f.tensor(i)["data"].size == n


# ---- the reference's reader tests (reader.rs:819-933)
def test_rejects_tensor_with_unknown_byte_layout():
    e = _err(_build([("unknown", (7,), 999, 0)], bytes(range(1, 8))))
    assert e.status == WLStatus.GGUF_PARSE
    assert "unsupported type" in e.message and "byte length is unknown" in e.message


def test_rejects_overlapping_known_tensors():
    e = _err(_build([("first", (2,), 0, 0), ("second", (1,), 0, 4)], bytes(8)))
    assert "overlaps next tensor" in e.message


def test_rejects_i2s_scale_block_overlapping_next_tensor():
    e = _err(_build([("i2s", (128,), 36, 0), ("next", (1,), 0, 48)], bytes(64)))
    assert "scale block ends" in e.message and "overlapping next tensor" in e.message


def test_rejects_shape_and_byte_length_overflow():
    assert "shape product overflow" in _err(_build([("bad", (2 ** 64 - 1, 2), 24, 0)], b"")).message
    assert "byte length overflow" in _err(_build([("bad", (2 ** 64 - 1,), 28, 0)], b"")).message


@pytest.mark.parametrize("shape,t,n,text", [((31,), 2, 0, "Q4_0 row length 31"),
                                            ((16, 2), 8, 34, "Q8_0 row length 16"),
                                            ((16, 2), 2, 18, "Q4_0 row length 16"),
                                            ((128, 2), 12, 144, "Q4_K row length 128")])
def test_rejects_incomplete_quantized_rows(shape, t, n, text):
    assert text in _err(_build([("bad", shape, t, 0)], bytes(n))).message


def test_rejects_excessive_header_counts_and_dims_and_arrays():
    e = _err(_header(1_000_001, 0))
    assert "tensor_count" in e.message and "safety limit" in e.message
    e = _err(_header(0, 1_000_001))
    assert "metadata_kv_count" in e.message and "safety limit" in e.message
    d = _header(1, 0) + gguf._s("bad") + struct.pack("<I", 5) + bytes(24)
    assert "n_dims 5 exceeds 4" in _err(d).message
    d = _header(0, 1) + gguf._s("array") + struct.pack("<IIQ", 9, 0, 1_000_001)
    e = _err(d)
    assert "array count" in e.message and "safety limit" in e.message


def test_error_classes():
    good = gguf.write_gguf({"k": 1}, [("t", (4,), 0, bytes(16))])
    assert _err(b"GGUX" + good[4:]).status == WLStatus.INVALID_MAGIC
    assert _err(good[:4] + struct.pack("<I", 1) + good[8:]).status == WLStatus.UNSUPPORTED_VERSION
    assert _err(good[:-20]).status == WLStatus.TENSOR_OUT_OF_BOUNDS  # cut into the tensor
    assert _err(good[:20]).status == WLStatus.GGUF_PARSE
    assert _err(_build([("a", (4,), 0, 0), ("b", (4,), 0, 0)], bytes(16))).status == \
        WLStatus.GGUF_PARSE  # shared offset
    bad_align = gguf.write_gguf({"general.alignment": (gguf.U32, 3)}, [])
    assert "invalid alignment" in _err(bad_align).message
    unknown_value = _header(0, 1) + gguf._s("k") + struct.pack("<I", 13)
    assert "unknown metadata value type" in _err(unknown_value).message


def test_model_config_errors_follow_the_reference():
    m = synth.bitnet_model(np.random.default_rng(4), n_layers=1, n_embd=256, n_heads=2,
                           n_kv_heads=1, n_ff=256, vocab=50, max_seq=8)

    def cfg_error(data):
        with pytest.raises(WillametteError) as e:
            gguf.GgufFile(data).model_config()
        return e.value

    b = gguf.bitnet_gguf(m)
    f = gguf.GgufFile(b)
    assert f.model_config()[1] == 0
    meta = {"general.architecture": "gpt2"}
    assert cfg_error(gguf.write_gguf(meta, [])).status == WLStatus.UNSUPPORTED_ARCHITECTURE
    meta = {"general.architecture": "bitnet-b1.58", "bitnet-b1.58.block_count": 1}
    assert cfg_error(gguf.write_gguf(meta, [])).status == WLStatus.MISSING_METADATA
    assert cfg_error(gguf.write_gguf({}, [])).status == WLStatus.MISSING_METADATA
    # rope.dimension_count must equal head_dim (config.rs:131-138)
    good = {"general.architecture": "bitnet", "bitnet.block_count": 1, "bitnet.embedding_length": 256,
            "bitnet.feed_forward_length": 256, "bitnet.context_length": 8,
            "bitnet.attention.head_count": 2, "bitnet.attention.head_count_kv": 1,
            "bitnet.attention.layer_norm_rms_epsilon": 1e-5, "bitnet.rope.dimension_count": 128,
            "bitnet.rope.freq_base": 500000.0, "bitnet.vocab_size": 50}
    assert gguf.GgufFile(gguf.write_gguf(good, [])).model_config()[0]["head_dim"] == 128
    bad = dict(good, **{"bitnet.rope.dimension_count": 64})
    assert cfg_error(gguf.write_gguf(bad, [])).status == WLStatus.GGUF_PARSE
    bad = dict(good, **{"bitnet.attention.head_count_kv": 3})
    assert cfg_error(gguf.write_gguf(bad, [])).status == WLStatus.GGUF_PARSE
    # llama: partial RoPE and RoPE scaling are not implemented (config.rs:196-220)
    lm = {"general.architecture": "llama", "llama.block_count": 1, "llama.embedding_length": 128,
          "llama.feed_forward_length": 256, "llama.context_length": 8,
          "llama.attention.head_count": 2, "llama.attention.layer_norm_rms_epsilon": 1e-5,
          "tokenizer.ggml.tokens": ["a", "b", "c"]}
    cfg, var = gguf.GgufFile(gguf.write_gguf(lm, [])).model_config()
    assert var == 1 and cfg["n_kv_heads"] == 2 and cfg["vocab"] == 3
    assert cfg_error(gguf.write_gguf(dict(lm, **{"llama.rope.dimension_count": 32}), [])).status \
        == WLStatus.NOT_IMPLEMENTED
    assert cfg_error(gguf.write_gguf(dict(lm, **{"llama.rope.scaling.type": "linear"}), [])).status \
        == WLStatus.NOT_IMPLEMENTED
    assert gguf.GgufFile(gguf.write_gguf(dict(lm, **{"llama.rope.scaling.type": "none"}), [])) \
        .model_config()[1] == 1
    no_tok = {k: v for k, v in lm.items() if k != "tokenizer.ggml.tokens"}
    assert cfg_error(gguf.write_gguf(no_tok, [])).status == WLStatus.MISSING_METADATA
