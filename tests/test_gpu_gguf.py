"""Engines built straight from GGUF files (wl_bitnet_create_from_gguf /
wl_llama_batch_create_from_gguf, the reference's ModelGraph::from_gguf,
src/model/graph.rs:95-240) decode exactly like the engines built from the
same tensors passed as arrays, and the file-level errors follow the
reference."""
import numpy as np
import pytest

from project_willamette_b200 import WillametteError, gguf, synth
from project_willamette_b200._abi import WLStatus

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("exact", [False, True])
def test_bitnet_from_gguf_equals_from_arrays(exact):
    from project_willamette_b200.bitnet import BitNet
    m = synth.bitnet_model(np.random.default_rng(31), n_layers=3, n_embd=512, n_heads=4,
                           n_kv_heads=2, n_ff=768, vocab=1000, max_seq=40)
    f = gguf.GgufFile(gguf.bitnet_gguf(m))
    prompt = np.random.default_rng(1).integers(0, 1000, 12)
    a = BitNet(m, exact=exact)
    b = BitNet.from_gguf(f, exact=exact)
    try:
        ia, ha = a.generate(prompt, 10, hiddens=True)
        ib, hb = b.generate(prompt, 10, hiddens=True)
        assert ia.tolist() == ib.tolist()
        assert np.array_equal(ha.view(np.uint32), hb.view(np.uint32))
    finally:
        a.close()
        b.close()


def test_llama_from_gguf_equals_from_arrays():
    from project_willamette_b200.llama import LlamaBatch
    m = synth.llama_q8_model(np.random.default_rng(32), n_layers=2, n_embd=192, n_heads=3,
                             n_kv_heads=1, n_ff=384, vocab=700, max_seq=48)
    f = gguf.GgufFile(gguf.llama_gguf(m))
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, 700, n) for n in (5, 9, 2)]
    a = LlamaBatch(m, 3)
    b = LlamaBatch.from_gguf(f, 3)
    try:
        ia, ha = a.generate(prompts, 6, hiddens=True)
        ib, hb = b.generate(prompts, 6, hiddens=True)
        assert ia.tolist() == ib.tolist()
        assert np.array_equal(ha.view(np.uint32), hb.view(np.uint32))
    finally:
        a.close()
        b.close()


def test_gguf_model_errors():
    from project_willamette_b200.bitnet import BitNet
    from project_willamette_b200.llama import LlamaBatch
    m = synth.bitnet_model(np.random.default_rng(33), n_layers=1, n_embd=256, n_heads=2,
                           n_kv_heads=1, n_ff=256, vocab=64, max_seq=16)
    data = bytearray(gguf.bitnet_gguf(m))
    f = gguf.GgufFile(bytes(data))
    with pytest.raises(WillametteError) as e:
        LlamaBatch.from_gguf(f, 1)  # a BitNet file is not a llama model
    assert e.value.status == WLStatus.INVALID_ARGUMENT
    # a non-finite I2_S scale is rejected (tensor.rs:278-309)
    t = f.tensor("blk.0.attn_k.weight")
    off = bytes(data).find(t["data"].tobytes()) + t["data"].size
    data[off:off + 4] = np.float32(np.inf).tobytes()
    with pytest.raises(WillametteError) as e:
        BitNet.from_gguf(gguf.GgufFile(bytes(data)))
    assert e.value.status == WLStatus.GGUF_PARSE
    # a missing layer tensor is MissingMetadata
    meta_only = gguf.write_gguf({k: v for k, v in [("general.architecture", "bitnet"),
                                                   ("bitnet.block_count", 1),
                                                   ("bitnet.embedding_length", 256),
                                                   ("bitnet.feed_forward_length", 256),
                                                   ("bitnet.context_length", 16),
                                                   ("bitnet.attention.head_count", 2),
                                                   ("bitnet.attention.head_count_kv", 1),
                                                   ("bitnet.attention.layer_norm_rms_epsilon", 1e-5),
                                                   ("bitnet.rope.dimension_count", 128),
                                                   ("bitnet.rope.freq_base", 500000.0),
                                                   ("bitnet.vocab_size", 64)]}, [])
    with pytest.raises(WillametteError) as e:
        BitNet.from_gguf(gguf.GgufFile(meta_only))
    assert e.value.status == WLStatus.MISSING_METADATA
    # a separate output.weight lm-head is not supported by the Llama engine
    lm = synth.llama_q8_model(np.random.default_rng(34), n_layers=1, n_embd=128, n_heads=2,
                              n_kv_heads=1, n_ff=256, vocab=50, max_seq=16)
    raw = gguf.llama_gguf(lm)
    f2 = gguf.GgufFile(raw)
    tensors = [(t["name"], t["shape"], t["type"], t["data"]) for t in f2.tensors()]
    tensors.append(("output.weight", (128, 50), gguf.GGML_Q8_0, f2.tensor("token_embd.weight")["data"]))
    meta = {"general.architecture": "llama", "llama.block_count": 1, "llama.embedding_length": 128,
            "llama.feed_forward_length": 256, "llama.context_length": 16,
            "llama.attention.head_count": 2, "llama.attention.head_count_kv": 1,
            "llama.attention.layer_norm_rms_epsilon": 1e-5,
            "tokenizer.ggml.tokens": [str(i) for i in range(50)]}
    with pytest.raises(WillametteError) as e:
        LlamaBatch.from_gguf(gguf.GgufFile(gguf.write_gguf(meta, tensors)), 1)
    assert e.value.status == WLStatus.NOT_IMPLEMENTED
