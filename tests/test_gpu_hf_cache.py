"""The Hugging Face cache adapter: compress on append, attend from the packed
bytes, dequantise for models that run their own attention."""
import math

import numpy as np
import pytest
import torch

import khtest as K
from kudahitam import ops
from kudahitam.hf_cache import KudahitamCache, KudahitamLayer, from_dynamic_cache

pytestmark = pytest.mark.gpu


def _kv(B, H, S, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16)
    return k, v


def test_append_matches_one_shot_compression_and_grows():
    B, H, D = 2, 2, 128
    k, v = _kv(B, H, 300 + 7, D, 0)
    layer = KudahitamLayer(D, 3, 4, initial_capacity=64)
    layer.append(k[:, :, :300], v[:, :, :300])
    for t in range(300, 307):  # decode steps, one token each
        layer.append(k[:, :, t:t + 1], v[:, :, t:t + 1])
    assert layer.get_seq_length() == 307 and layer.k.capacity >= 307
    full = ops.compress(k, layer.d_k, layer.c)
    got = layer.k._first_rows()
    for name in ("code", "res", "norms", "rnorms"):
        assert torch.equal(getattr(got, name), getattr(full, name)), name
    layer.crop(-7)
    assert layer.get_seq_length() == 300


def test_attend_equals_decode_over_the_same_rows_with_gqa():
    B, Hk, n_q, D, S = 2, 2, 3, 128, 1500
    k, v = _kv(B, Hk, S, D, 1)
    layer = KudahitamLayer(D, 5, 6, initial_capacity=4000)  # capacity > length
    layer.append(k, v)
    q = torch.randn(B, Hk * n_q, D, device="cuda")
    got = layer.attend(q, n_splits=2)
    pk, pv = ops.compress(k, layer.d_k, layer.c), ops.compress(v, layer.d_v, layer.c)
    want = ops.decode_attention(q.view(B * Hk, n_q, D), pk, pv, layer.d_k, layer.d_v, layer.c,
                                n_splits=2)
    assert torch.equal(got, want.view(B, Hk * n_q, D))


def test_dequantized_path_reproduces_scores_and_decode():
    B, Hk, D, S = 1, 2, 128, 700
    k, v = _kv(B, Hk, S, D, 2)
    layer = KudahitamLayer(D, 7, 8)
    kh, vh = layer.update(k, v)
    assert kh.shape == (B, Hk, S, D) and kh.dtype == torch.bfloat16
    layer32 = KudahitamLayer(D, 7, 8)
    layer32.append(k, v)
    kf = layer32.k.dequantize(layer32.d_k, layer32.c, 1.0, torch.float32)
    vf = layer32.v.dequantize(layer32.d_v, layer32.c, math.sqrt(2 / math.pi), torch.float32)
    q = torch.randn(B, Hk, 1, D, device="cuda")
    sc = layer32.scores(q)  # the reference's estimator on the packed cache
    dot = torch.einsum("bhnd,bhsd->bhns", q, kf)
    for h in range(Hk):
        assert K.normwise(dot[0, h, 0].cpu().numpy(), sc[0, h, 0].cpu().numpy()) < 1e-5
    p = torch.softmax(dot / math.sqrt(D), dim=-1)
    att = torch.einsum("bhns,bhsd->bhnd", p, vf)[:, :, 0]
    got = layer32.attend(q[:, :, 0])
    for h in range(Hk):
        assert K.normwise(got[0, h].cpu().numpy(), att[0, h].cpu().numpy()) < 1e-4


def test_cache_object_and_dynamic_cache_conversion():
    from transformers import DynamicCache
    D = 128
    dc = DynamicCache()
    kvs = [_kv(1, 2, 200, D, 10 + l) for l in range(3)]
    for l, (k, v) in enumerate(kvs):
        dc.update(k, v, l)
    cache = from_dynamic_cache(dc)
    assert len(cache.layers) == 3 and cache.get_seq_length() == 200
    for l, (k, v) in enumerate(kvs):
        layer = cache.layers[l]
        ref = ops.compress(k, layer.d_k, layer.c)
        assert torch.equal(layer.k._first_rows().code, ref.code)
    # the Cache.update contract used by transformers models
    k1, v1 = _kv(1, 2, 1, D, 99)
    kk, vv = cache.update(k1, v1, 0)
    assert kk.shape == (1, 2, 201, D) and cache.get_seq_length(0) == 201
    assert cache.nbytes() < sum(k.numel() * 2 * 2 for k, _ in kvs) / 5


def test_generate_with_a_tiny_model():
    """A randomly initialised Llama-architecture model generates through the
    compressed cache (transformers calls update(); attention runs on the
    dequantised K / V) and stays close to the uncompressed run."""
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=2, num_key_value_heads=1, head_dim=128,
                                   vocab_size=512, max_position_embeddings=4096)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).cuda().to(torch.bfloat16).eval()
    ids = torch.randint(0, 512, (1, 300), device="cuda")
    with torch.no_grad():
        ref = model(ids, use_cache=True).logits[:, -1].float()
        cache = KudahitamCache(head_dim=128)
        out = model(ids, past_key_values=cache, use_cache=True)
        got = out.logits[:, -1].float()
        assert cache.get_seq_length() == 300
        cos = torch.nn.functional.cosine_similarity(ref, got).item()
        assert cos > 0.9, cos
        gen = model.generate(ids[:, :50], past_key_values=KudahitamCache(head_dim=128),
                             max_new_tokens=5, do_sample=False)
        assert gen.shape == (1, 55)


def test_generate_attends_from_the_packed_cache(monkeypatch):
    """With attn_implementation="kudahitam" and packed_attention=True, every
    decode step of generate() attends from the packed bytes through the
    decode kernel: the cache is never dequantised (counted), prefill
    attends to the prompt exactly, and the logits stay close to an
    uncompressed run of the same model."""
    transformers = pytest.importorskip("transformers")
    from kudahitam import hf_cache
    name = hf_cache.register_attention()
    cfg = transformers.LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                                   vocab_size=512, max_position_embeddings=4096)
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(cfg).cuda().to(torch.bfloat16).eval()
    ref_model = transformers.LlamaForCausalLM(cfg).cuda().to(torch.bfloat16).eval()
    ref_model.load_state_dict(model.state_dict())
    model.set_attn_implementation(name)
    calls = {"dequantize": 0, "attend": 0}
    real_deq, real_attend = hf_cache.PackedSeq.dequantize, hf_cache.KudahitamLayer.attend

    def deq(self, *a, **k):
        calls["dequantize"] += 1
        return real_deq(self, *a, **k)

    def att(self, *a, **k):
        calls["attend"] += 1
        return real_attend(self, *a, **k)

    monkeypatch.setattr(hf_cache.PackedSeq, "dequantize", deq)
    monkeypatch.setattr(hf_cache.KudahitamLayer, "attend", att)
    ids = torch.randint(0, 512, (1, 400), device="cuda")
    new = 8
    with torch.no_grad():
        cache = hf_cache.KudahitamCache(head_dim=128, packed_attention=True)
        gen = model.generate(ids, past_key_values=cache, max_new_tokens=new, do_sample=False,
                             min_new_tokens=new)
        assert gen.shape == (1, 400 + new)
        assert calls["dequantize"] == 0
        assert calls["attend"] == 2 * (new - 1)  # every decode step of both layers
        # one more step by hand: logits from the packed cache vs uncompressed
        logits = model(gen[:, -1:], past_key_values=cache, use_cache=True).logits[:, -1].float()
        full = ref_model(gen, use_cache=False).logits[:, -1].float()
        cos = torch.nn.functional.cosine_similarity(full, logits).item()
        assert cos >= 0.9, cos
        assert calls["dequantize"] == 0
