"""A decoder loaded from a GGUF v3 file (beacon_cuda_model_load_gguf) against
the oracle engine built from the same tensor bytes.

The file follows real GGUF conventions: Q4_0 nibbles in the split order
(byte i -> elements i, i + 16), mixed block types across tensors as quantized
releases mix them (Q4_0, Q8_0, Q4_K, Q5_K, Q6_K), f32 norm weights, and
either an f16 embedding with its own output tensor or a quantized embedding
tied as the output (weights.rs:116-166 name mapping).
"""
import numpy as np
import pytest

import oracle as orc
from gguf_writer import GgufBuilder, llama_kv

pytestmark = pytest.mark.gpu

H, LAYERS, HEADS, KV_HEADS, FFN, VOCAB = 256, 2, 4, 2, 512, 300
HD = H // HEADS
ORC_TYPE = {"Q4_0": orc.Q4_0, "Q8_0": orc.Q8_0, "Q4_K": orc.Q4_K, "Q5_K": orc.Q5_K, "Q6_K": orc.Q6_K,
            "F16": orc.F16, "F32": orc.F32}


@pytest.fixture(scope="module")
def be(cuda_lib):
    from beacon_cuda import CudaBackend
    return CudaBackend(0)


def sane_blocks(rng, t, n, k, scale=0.001):
    from test_gpu_formats import sane_blocks as sb
    return sb(rng, ORC_TYPE[t], n, k, scale)


# q/k/v share one fused tile and gate/up another, so each group has one block type
KINDS = {"attn_q": "Q4_0", "attn_k": "Q4_0", "attn_v": "Q4_0", "attn_output": "Q4_K", "ffn_gate": "Q5_K",
         "ffn_up": "Q5_K", "ffn_down": "Q6_K"}


def build(tmp_path, quantized_embedding: bool, kinds=None, name=None):
    rng = np.random.default_rng(7 + quantized_embedding)
    b = llama_kv(GgufBuilder(), H, LAYERS, HEADS, KV_HEADS, FFN, VOCAB)
    tensors = []   # (name, shape, type, data)

    def lin(name, n, k, t):
        if t in ("Q4_0", "Q8_0", "Q4_K"):   # the fixture quantizer; Q4_0 in the GGUF split order
            data = orc.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), ORC_TYPE[t],
                                orc.NIBBLE_GGUF_SPLIT)
        else:
            data = sane_blocks(rng, t, n, k)
        tensors.append((name, (n, k), t, data))

    if quantized_embedding:
        lin("token_embd.weight", VOCAB, H, "Q8_0")     # tied: no output.weight
    else:
        tensors.append(("token_embd.weight", (VOCAB, H), "F16", rng.standard_normal((VOCAB, H)).astype(np.float16)))
        lin("output.weight", VOCAB, H, "Q6_K")
    tensors.append(("output_norm.weight", (H,), "F32", (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)))
    kinds = dict(KINDS, **(kinds or {}))
    for li in range(LAYERS):
        p = f"blk.{li}."
        tensors.append((p + "attn_norm.weight", (H,), "F32", (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)))
        tensors.append((p + "ffn_norm.weight", (H,), "F32", (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)))
        lin(p + "attn_q.weight", HEADS * HD, H, kinds["attn_q"])
        lin(p + "attn_k.weight", KV_HEADS * HD, H, kinds["attn_k"])
        lin(p + "attn_v.weight", KV_HEADS * HD, H, kinds["attn_v"])
        lin(p + "attn_output.weight", H, HEADS * HD, kinds["attn_output"])
        lin(p + "ffn_gate.weight", FFN, H, kinds["ffn_gate"])
        lin(p + "ffn_up.weight", FFN, H, kinds["ffn_up"])
        lin(p + "ffn_down.weight", H, FFN, kinds["ffn_down"])
    for name, shape, t, data in tensors:
        b.add_tensor(name, shape, t, data)
    return b.write(tmp_path / (name or ("q.gguf" if quantized_embedding else "f.gguf"))), tensors


def oracle_from(tensors, rtz):
    c = orc.OracleModelConfig(VOCAB, H, LAYERS, HEADS, KV_HEADS, HD, FFN, 32, weights_rtz=rtz)
    om = orc.OracleModel(c)
    slot = {"attn_norm": orc.W_ATTN_NORM, "attn_q": orc.W_Q, "attn_k": orc.W_K, "attn_v": orc.W_V,
            "attn_output": orc.W_O, "ffn_norm": orc.W_FFN_NORM, "ffn_gate": orc.W_GATE, "ffn_up": orc.W_UP,
            "ffn_down": orc.W_DOWN}
    names = {name for name, *_ in tensors}
    for name, shape, t, data in tensors:
        if name == "token_embd.weight":
            om.set_weight(0, orc.W_EMBED, data, ORC_TYPE[t], orc.NIBBLE_GGUF_SPLIT)
            if "output.weight" not in names:
                om.set_weight(0, orc.W_LM_HEAD, data, ORC_TYPE[t], orc.NIBBLE_GGUF_SPLIT)
        elif name == "output.weight":
            om.set_weight(0, orc.W_LM_HEAD, data, ORC_TYPE[t], orc.NIBBLE_GGUF_SPLIT)
        elif name == "output_norm.weight":
            om.set_weight(0, orc.W_FINAL_NORM, data, ORC_TYPE[t])
        else:
            _, li, part, _ = name.split(".")
            om.set_weight(int(li), slot[part], data, ORC_TYPE[t], orc.NIBBLE_GGUF_SPLIT)
    return om


@pytest.mark.parametrize("quantized_embedding", [False, True])
def test_decoder_loaded_from_gguf_matches_oracle(be, tmp_path, quantized_embedding):
    from beacon_cuda import CudaModel, DecoderConfig
    from beacon_cuda import _lib as L
    from beacon_cuda.gguf import GgufFile
    path, tensors = build(tmp_path, quantized_embedding)
    f = GgufFile(path)
    cfg = f.model_config(max_context=32)
    assert (cfg["vocab_size"], cfg["hidden_size"], cfg["num_layers"], cfg["head_dim"]) == (VOCAB, H, LAYERS, HD)
    # the f16 / exact pair compares unrounded weights; the quantized embedding
    # is stored as f16 values, so that pair runs the CPU-reproducing numerics
    numerics = L.NUMERICS_REF_RTZ if quantized_embedding else L.NUMERICS_EXACT
    m = CudaModel(be, DecoderConfig(**cfg, numerics=numerics, kv_dtype=L.DTYPE_F32))
    m.load_gguf(f)
    om = oracle_from(tensors, rtz=quantized_embedding)
    tol = 1e-4 if quantized_embedding else 1e-3
    prompt = [1, 17, 255, 3, 299, 42]
    assert np.abs(m.forward(prompt, 0) - om.forward(prompt, 0)).max() <= tol
    tok, pos = 9, len(prompt)
    for _ in range(4):
        nxt, lg = m.decode_step([tok], pos, want_logits=True)
        assert np.abs(lg[0] - om.forward([tok], pos)[0]).max() <= tol
        tok, pos = int(nxt[0]), pos + 1
    m.close()
    f.close()


def test_load_gguf_reports_missing_and_misshapen_tensors(be, tmp_path):
    from beacon_cuda import CudaModel, DecoderConfig, EngineError, ShapeMismatch
    from beacon_cuda.gguf import GgufFile
    path, tensors = build(tmp_path, False)
    f = GgufFile(path)
    cfg = f.model_config(max_context=16)
    m = CudaModel(be, DecoderConfig(**dict(cfg, intermediate_size=FFN * 2)))
    with pytest.raises(ShapeMismatch):          # ffn tensors disagree with the model
        m.load_gguf(f)
    b = llama_kv(GgufBuilder(), H, LAYERS, HEADS, KV_HEADS, FFN, VOCAB)
    for name, shape, t, data in tensors:
        if name != "blk.1.ffn_up.weight":
            b.add_tensor(name, shape, t, data)
    g = GgufFile(b.write(tmp_path / "missing.gguf"))
    m2 = CudaModel(be, DecoderConfig(**g.model_config(max_context=16)))
    with pytest.raises(EngineError, match="blk.1.ffn_up.weight"):
        m2.load_gguf(g)


def test_load_gguf_refuses_mixed_qkv_block_types(be, tmp_path):
    """q/k/v share one tile layout: a file whose attn_v has another block type
    than attn_q is refused (UNSUPPORTED_DTYPE) instead of being misread."""
    from beacon_cuda import CudaModel, DecoderConfig, EngineError
    from beacon_cuda import _lib as L
    from beacon_cuda.gguf import GgufFile
    path, _ = build(tmp_path, False, kinds={"attn_v": "Q8_0"}, name="mixed.gguf")
    f = GgufFile(path)
    m = CudaModel(be, DecoderConfig(**f.model_config(max_context=16)))
    with pytest.raises(EngineError) as e:
        m.load_gguf(f)
    assert e.value.status == L.ERR_UNSUPPORTED_DTYPE and "blk.0.attn_v.weight" in str(e.value)
