"""The PyTorch restatement of the reference's decode step (neokernel_b200/qwen3.py) pinned to
transformers' own Qwen3 modules, on the CPU.

Every fused CUDA kernel of the decode step is checked on the GPU against ``qwen3.layer_step``
and ``qwen3.decode_step``; these tests pin those two to the modules the reference's own test
compares its Triton layer with (tests/test_hand_rolled_kernels.py:148-180 in the reference:
``Qwen3DecoderLayer`` on the Qwen3-4B widths, ``normal_(0, .02)`` weights, seed 714, batches
1/4/16, a 512-position cache prefix, atol .125 / rtol .03), and to ``Qwen3ForCausalLM`` for the
embedding, final norm, lm_head and greedy choice over a multi-step decode.
"""

import types

import pytest
import torch
from transformers import DynamicCache, Qwen3Config
from transformers.models.qwen3.modeling_qwen3 import (Qwen3DecoderLayer, Qwen3ForCausalLM,
                                                      Qwen3RotaryEmbedding)

from neokernel_b200 import qwen3


def pack_layer(native):
    """The reference's LayerWeights packing (engine/kernels/weights.py:10-29) of an HF layer."""
    a, m = native.self_attn, native.mlp
    lw = types.SimpleNamespace()
    lw.qkv_weight = torch.cat((a.q_proj.weight, a.k_proj.weight, a.v_proj.weight)).detach()
    lw.gate_up_weight = torch.cat((m.gate_proj.weight, m.up_proj.weight)).detach()
    lw.o_weight = a.o_proj.weight.detach()
    lw.down_weight = m.down_proj.weight.detach()
    lw.qkv, lw.gate_up = lw.qkv_weight.t(), lw.gate_up_weight.t()
    lw.o, lw.down = lw.o_weight.t(), lw.down_weight.t()
    lw.input_norm = native.input_layernorm.weight.detach()
    lw.post_norm = native.post_attention_layernorm.weight.detach()
    lw.q_norm, lw.k_norm = a.q_norm.weight.detach(), a.k_norm.weight.detach()
    return lw


def dims_of(config, layers=1):
    return qwen3.Qwen3Dims(config.hidden_size, config.intermediate_size,
                           config.num_attention_heads, config.num_key_value_heads,
                           config.head_dim, layers, config.vocab_size, config.rms_norm_eps,
                           config.rope_parameters["rope_theta"], config.tie_word_embeddings)


CONFIG_4B_LAYER = dict(hidden_size=2560, intermediate_size=9728, num_attention_heads=32,
                       num_key_value_heads=8, head_dim=128, num_hidden_layers=1, rope_theta=5e6,
                       rms_norm_eps=1e-6, vocab_size=64)


def test_rope_tables_match_transformers():
    config = Qwen3Config(**CONFIG_4B_LAYER)
    rotary = Qwen3RotaryEmbedding(config)
    cap = 2080
    cos, sin = rotary(torch.empty(1, dtype=torch.bfloat16), torch.arange(cap)[None])
    ours_cos, ours_sin = qwen3.rope_tables(dims_of(config), cap, "cpu")
    assert torch.equal(ours_cos, cos[0]) and torch.equal(ours_sin, sin[0])


@pytest.mark.parametrize("gains", ("ones", "random"))
@torch.inference_mode()
def test_layer_step_matches_transformers_decoder_layer(gains):
    """The reference's test_layer_all_switch_combinations, with qwen3.layer_step (linears on
    torch.mm, as the reference calls them) in place of DecodeBuffers.layer."""
    config = Qwen3Config(**CONFIG_4B_LAYER)
    config._attn_implementation = "sdpa"
    torch.manual_seed(714)
    native = Qwen3DecoderLayer(config, 0).bfloat16().eval()
    for name, p in native.named_parameters():
        if "norm" not in name:
            p.normal_(0, .02)
        elif gains == "random":
            p.uniform_(0.5, 1.5)
    lw = pack_layer(native)
    d = dims_of(config)
    rotary = Qwen3RotaryEmbedding(config)
    capacity, pos = 640, 512
    cos, sin = rotary(torch.empty(1, dtype=torch.bfloat16), torch.arange(capacity)[None])
    for batch in (1, 4, 16):
        x = torch.randn(batch, 1, d.hidden).to(torch.bfloat16)
        prefix_k = torch.randn(batch, d.kv_heads, pos, d.head_dim).to(torch.bfloat16)
        prefix_v = torch.randn(batch, d.kv_heads, pos, d.head_dim).to(torch.bfloat16)
        position = torch.tensor([pos])
        cache = DynamicCache()
        cache.update(prefix_k, prefix_v, 0)
        ref = native(x, attention_mask=None, position_ids=position[None], past_key_values=cache,
                     use_cache=True, position_embeddings=(cos[:, pos:pos + 1], sin[:, pos:pos + 1]))
        ref = ref[0] if isinstance(ref, tuple) else ref

        st = qwen3.DecodeState(types.SimpleNamespace(dims=d, layers=[lw]), batch, capacity, "cpu")
        k_cache, v_cache = st.k_cache[0], st.v_cache[0]
        k_cache[:, :, :pos].copy_(prefix_k)
        v_cache[:, :, :pos].copy_(prefix_v)
        st.x.copy_(x[:, 0])
        st.position.fill_(pos)
        qwen3.layer_step(st, lw, k_cache, v_cache, d, torch.mm)
        diff = (st.x.float() - ref[:, 0].float()).abs().max().item()
        torch.testing.assert_close(st.x.float(), ref[:, 0].float(), atol=.125, rtol=.03,
                                   msg=f"layer/{batch}/{gains}: max |diff| {diff}")
        print(f"layer/{batch}/{gains}: max |diff| {diff}")
        # the new K/V slot is the layer's own: RoPE'd normalised key, raw value
        kv = cache.layers[0]
        torch.testing.assert_close(k_cache[:, :, pos].float(), kv.keys[:, :, pos].float(),
                                   atol=.0625, rtol=.01)
        assert torch.equal(v_cache[:, :, pos], kv.values[:, :, pos])


def tiny_model(init, seed=3):
    """A small untied Qwen3 (2 layers, hidden 512, 4 query / 2 KV heads of 128, vocab 1000) with
    qwen3.Qwen3Weights' draws loaded into transformers' Qwen3ForCausalLM."""
    config = Qwen3Config(hidden_size=512, intermediate_size=1024, num_attention_heads=4,
                         num_key_value_heads=2, head_dim=128, num_hidden_layers=2,
                         rope_theta=1e6, rms_norm_eps=1e-6, vocab_size=1000,
                         tie_word_embeddings=False)
    config._attn_implementation = "sdpa"
    d = dims_of(config, layers=2)
    w = qwen3.Qwen3Weights(d, seed=seed, device="cpu", init=init)
    model = Qwen3ForCausalLM(config).bfloat16().eval()
    D = d.head_dim
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(w.embed)
        model.lm_head.weight.copy_(w.lm_head_weight)
        model.model.norm.weight.copy_(w.final_norm)
        for layer, lw in zip(model.model.layers, w.layers):
            a, m = layer.self_attn, layer.mlp
            q_end, k_end = d.heads * D, d.heads * D + d.kv_heads * D
            a.q_proj.weight.copy_(lw.qkv_weight[:q_end])
            a.k_proj.weight.copy_(lw.qkv_weight[q_end:k_end])
            a.v_proj.weight.copy_(lw.qkv_weight[k_end:])
            a.o_proj.weight.copy_(lw.o_weight)
            m.gate_proj.weight.copy_(lw.gate_up_weight[:d.intermediate])
            m.up_proj.weight.copy_(lw.gate_up_weight[d.intermediate:])
            m.down_proj.weight.copy_(lw.down_weight)
            layer.input_layernorm.weight.copy_(lw.input_norm)
            layer.post_attention_layernorm.weight.copy_(lw.post_norm)
            a.q_norm.weight.copy_(lw.q_norm)
            a.k_norm.weight.copy_(lw.k_norm)
    return d, w, model


@pytest.mark.parametrize("init", qwen3.INITS)
@torch.inference_mode()
def test_decode_step_matches_transformers_causal_lm(init):
    """qwen3.decode_step token by token against Qwen3ForCausalLM with a growing cache, both fed
    transformers' greedy tokens: logits within the layer test's tolerance at every step, and —
    with the decisive init — the same greedy choice at every step."""
    d, w, model = tiny_model(init)
    B, prompt_len, new = 2, 4, 20
    gen = torch.Generator().manual_seed(11)
    prompt = torch.randint(0, d.vocab, (B, prompt_len), generator=gen)
    cap = prompt_len + new
    st = qwen3.DecodeState(w, B, cap, "cpu")
    cache = DynamicCache()
    tok = prompt[:, 0].clone()
    margins, out_ours, out_hf = [], [], []
    for i in range(prompt_len + new - 1):
        if i < prompt_len:
            tok = prompt[:, i]
        # both models take the same token (transformers' greedy choice), so a near-tie flip
        # under the flat init cannot send them down different sequences
        st.tokens.copy_(tok)
        st.position.fill_(i)
        qwen3.decode_step(st, w, torch.mm)
        logits = model(input_ids=tok[:, None], past_key_values=cache, use_cache=True,
                       position_ids=torch.full((B, 1), i), cache_position=torch.tensor([i])).logits[:, 0]
        torch.testing.assert_close(st.logits.float(), logits.float(), atol=.125, rtol=.03,
                                   msg=f"step {i} ({init})")
        top2 = logits.float().topk(2, dim=-1).values
        margins.append((top2[:, 0] - top2[:, 1]).min().item())
        if i >= prompt_len - 1:
            nxt_ours, nxt_hf = st.next_tokens.clone(), logits.argmax(-1)
            out_ours.append(nxt_ours)
            out_hf.append(nxt_hf)
            tok = nxt_hf
    print(f"decode/{init}: smallest top-2 margin per step {[round(m, 3) for m in margins]}")
    if init == "decisive":
        assert torch.equal(torch.stack(out_ours), torch.stack(out_hf))
        assert min(margins[prompt_len - 1:]) > 4.0, margins
