"""The drop-in on real transformers models: tiny random-init OLMoE and Qwen3-Next decoders (the two
families moelab loads, moelab/loader.py:53-65, 211-223) run stock, then with ``moeb200.install()``
swapping every MoE block's ``experts`` for B200Experts and its ``gate`` for B200Router.

* install with fp16 records ("hi"): logits within tolerance of the stock model; greedy decoding
  with the KV cache (prefill, then one-token decode calls) gives the stock model's tokens, up to a
  position where the stock model itself had a near-tie;
* install with int4 records ("lo"): the same against the stock model whose expert weights are
  replaced by the records' dequantised values (the oracle's materialize_f32);
* B200Router.from_module on every block: the same top-k experts and weights as the stock router;
* ``runtime.capture_hook`` sees every expert call of a forward (moelab's segmented-graph hook,
  moelab/runtime.py:1094-1112) and its result is what the model uses.

Tolerances: the stock model rounds each expert's gate/up and down products to fp16; the B200
kernels accumulate the layer in fp32 and round once, so logits agree to a few 1e-3 relative."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

import moeb200
from moeb200 import ops
from moeb200.runtime import B200Experts, B200Router, iter_moe_blocks
from oracle import moe_oracle as O

pytestmark = pytest.mark.gpu

V = 512
LOGIT_TOL = 3e-2


def _tiny(family: str, seed: int):
    from transformers import OlmoeConfig, OlmoeForCausalLM, Qwen3NextConfig, Qwen3NextForCausalLM

    torch.manual_seed(seed)
    if family == "olmoe":
        cfg = OlmoeConfig(vocab_size=V, hidden_size=256, intermediate_size=128, num_hidden_layers=2,
                          num_attention_heads=4, num_key_value_heads=4, num_experts=16, num_experts_per_tok=4,
                          norm_topk_prob=False, max_position_embeddings=128)
        model = OlmoeForCausalLM(cfg)
    else:
        cfg = Qwen3NextConfig(vocab_size=V, hidden_size=256, intermediate_size=256, moe_intermediate_size=128,
                              shared_expert_intermediate_size=128, num_hidden_layers=4, num_attention_heads=4,
                              num_key_value_heads=2, head_dim=64, linear_num_value_heads=4, linear_num_key_heads=2,
                              linear_key_head_dim=32, linear_value_head_dim=32, num_experts=16,
                              num_experts_per_tok=4, decoder_sparse_step=1, mlp_only_layers=[],
                              max_position_embeddings=128)
        model = Qwen3NextForCausalLM(cfg)
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for _, blk in iter_moe_blocks(model):
            # spread the router logits so that top-k has no near-ties at random init
            blk.gate.weight.copy_(torch.randn(blk.gate.weight.shape, generator=g) * 0.1)
            blk.experts.gate_up_proj.copy_(torch.randn(blk.experts.gate_up_proj.shape, generator=g) * 0.05)
            blk.experts.down_proj.copy_(torch.randn(blk.experts.down_proj.shape, generator=g) * 0.05)
    return model.eval()


def _logits(model, ids):
    with torch.no_grad():
        return model(ids).logits.float()


def _greedy(model, ids, n):
    with torch.no_grad():
        return model.generate(ids, max_new_tokens=n, min_new_tokens=n, do_sample=False, use_cache=True,
                              pad_token_id=0, eos_token_id=None)


def _check_tokens_agree(stock, ours_seq, ref_seq, n_prompt, tol_abs):
    """Greedy sequences agree, or first differ where the stock model's top-2 gap is within the
    logit tolerance (a near-tie, not a wrong expert sum)."""
    ours_seq, ref_seq = ours_seq[0].tolist(), ref_seq[0].tolist()
    for p in range(n_prompt, len(ref_seq)):
        if ours_seq[p] != ref_seq[p]:
            lg = _logits(stock, torch.tensor([ref_seq[:p]], device=next(stock.parameters()).device))[0, -1]
            top2 = torch.topk(lg, 2).values
            assert float(top2[0] - top2[1]) <= 2 * tol_abs, (p, ours_seq, ref_seq)
            return
    assert ours_seq == ref_seq


def _moe_modules(model):
    """The model's MoE blocks in layer order (stock sparse blocks or their B200 replacements)."""
    return [m for m in model.modules() if type(m).__name__.endswith("SparseMoeBlock") or type(m).__name__ == "B200MoeBlock"]


def _check_blocks_teacher_forced(ref_model, ours, ids, tol=1e-2):
    """Every MoE block of ours, fed the hidden states the reference model's block saw, gives that
    block's output within tol (no error carried from earlier layers, no routing flip from them)."""
    seen = []
    hooks = [b.register_forward_hook(lambda m, i, o: seen.append((i[0].detach(), o.detach())))
             for b in _moe_modules(ref_model)]
    try:
        _logits(ref_model, ids)
    finally:
        for h in hooks:
            h.remove()
    mine = _moe_modules(ours)
    assert len(mine) == len(seen)
    for li, (blk, (x, y)) in enumerate(zip(mine, seen)):
        with torch.no_grad():
            got = blk(x)
        got = got[0] if isinstance(got, tuple) else got
        err = float((got.float() - y.float()).abs().max() / y.float().abs().max())
        assert err < tol, (li, err)


def _check_logits(got, ref):
    """End to end: logits within LOGIT_TOL at (nearly) every position. A token whose routing sits on
    a near-tie in some layer may take the other expert after the tiny differences of earlier
    layers; that is allowed at no more than one position in eight."""
    scale = float(ref.abs().max())
    per_pos = (got - ref).abs().amax(-1) / scale
    bad = int((per_pos >= LOGIT_TOL).sum())
    assert bad <= per_pos.numel() // 8, (bad, float(per_pos.max()))


def _dequantised_stock(stock, rt, prec):
    """A copy of the stock model whose expert weights are the dequantised records of `prec`."""
    m = copy.deepcopy(stock)
    lay = rt.layouts[prec]
    with torch.no_grad():
        for li, blk in iter_moe_blocks(m):
            for e in range(blk.experts.gate_up_proj.shape[0]):
                gu, dn = O.materialize_f32(lay, rt.record(li, e, prec).cpu().numpy())
                blk.experts.gate_up_proj[e].copy_(torch.from_numpy(gu))
                blk.experts.down_proj[e].copy_(torch.from_numpy(dn))
    return m


@pytest.mark.parametrize("family", ["olmoe", "qwen3_next"])
@pytest.mark.parametrize("prec", ["fp16", "int4"])
def test_install_matches_stock_model(cuda_dev, family, prec):
    stock = _tiny(family, seed=7).to(cuda_dev, torch.float16)
    gen = torch.Generator().manual_seed(3)
    ids = torch.randint(0, V, (2, 16), generator=gen).to(cuda_dev)
    ours = copy.deepcopy(stock)
    policy = ops.PolicySpec("hi" if prec == "fp16" else "lo")
    blocks = [b for _, b in iter_moe_blocks(ours)]
    rt = moeb200.install(ours, [prec], policy)
    assert blocks and all(isinstance(b.experts, B200Experts) and isinstance(b.gate, B200Router) for b in blocks)
    ref_model = stock if prec == "fp16" else _dequantised_stock(stock, rt, prec)

    _check_blocks_teacher_forced(ref_model, ours, ids)
    ref = _logits(ref_model, ids)
    got = _logits(ours, ids)
    _check_logits(got, ref)
    assert int(rt.miss.item()) == 0

    prompt = ids[:1, :8]
    tol_abs = LOGIT_TOL * float(ref.abs().max())
    _check_tokens_agree(ref_model, _greedy(ours, prompt, 12), _greedy(ref_model, prompt, 12), 8, tol_abs)


@pytest.mark.parametrize("prec", ["fp16", "int4"])
def test_install_with_folded_shared_expert_matches_stock(cuda_dev, prec):
    # Qwen3-Next blocks replaced whole: the shared expert runs as expert E in the routed launches
    from moeb200.runtime import B200MoeBlock

    stock = _tiny("qwen3_next", seed=7).to(cuda_dev, torch.float16)
    ids = torch.randint(0, V, (2, 16), generator=torch.Generator().manual_seed(3)).to(cuda_dev)
    ours = copy.deepcopy(stock)
    rt = moeb200.install(ours, [prec], ops.PolicySpec("hi" if prec == "fp16" else "lo"), fold_shared=True)
    folded = [m for m in ours.modules() if isinstance(m, B200MoeBlock)]
    assert len(folded) == 4 and rt.num_experts == 17
    ref_model = stock
    if prec == "int4":  # the stock model with the routed and shared MLPs at their int4 values
        ref_model = _dequantised_stock(stock, rt, prec)
        lay = rt.layouts[prec]
        with torch.no_grad():
            for li, blk in iter_moe_blocks(ref_model):
                gu, dn = O.materialize_f32(lay, rt.record(li, 16, prec).cpu().numpy())
                I = gu.shape[0] // 2
                blk.shared_expert.gate_proj.weight.copy_(torch.from_numpy(gu[:I]))
                blk.shared_expert.up_proj.weight.copy_(torch.from_numpy(gu[I:]))
                blk.shared_expert.down_proj.weight.copy_(torch.from_numpy(dn))
    _check_blocks_teacher_forced(ref_model, ours, ids)
    ref = _logits(ref_model, ids)
    got = _logits(ours, ids)
    _check_logits(got, ref)
    assert int(rt.miss.item()) == 0
    tol_abs = LOGIT_TOL * float(ref.abs().max())
    prompt = ids[:1, :8]
    _check_tokens_agree(ref_model, _greedy(ours, prompt, 12), _greedy(ref_model, prompt, 12), 8, tol_abs)


@pytest.mark.parametrize("family", ["olmoe", "qwen3_next"])
def test_router_from_module_matches_stock_router(cuda_dev, family):
    stock = _tiny(family, seed=11).to(cuda_dev, torch.float16)
    h = torch.randn(64, 256, generator=torch.Generator().manual_seed(5)).to(cuda_dev, torch.float16)
    for _, blk in iter_moe_blocks(stock):
        p_ref, w_ref, i_ref = blk.gate(h)
        r = B200Router.from_module(blk.gate).to(cuda_dev)
        assert (r.top_k, r.num_experts, r.norm_topk_prob) == (blk.gate.top_k, blk.gate.num_experts,
                                                            bool(blk.gate.norm_topk_prob))
        p, w, i = r(h)
        assert torch.allclose(p, p_ref.float(), rtol=2e-3, atol=1e-5)
        # identical expert choice wherever the stock k-th / (k+1)-th probabilities are apart
        srt = torch.sort(p_ref.float(), dim=-1, descending=True).values
        clear = (srt[:, r.top_k - 1] - srt[:, r.top_k]) > 1e-3
        assert int(clear.sum()) > 48
        assert torch.equal(torch.sort(i[clear], -1).values, torch.sort(i_ref[clear], -1).values)
        assert torch.allclose(w[clear], w_ref.float()[clear], rtol=2e-3, atol=1e-5)


def test_capture_hook_sees_every_expert_call(cuda_dev):
    stock = _tiny("olmoe", seed=13).to(cuda_dev, torch.float16)
    ours = copy.deepcopy(stock)
    rt = moeb200.install(ours, ["fp16"])
    ids = torch.randint(0, V, (1, 10), generator=torch.Generator().manual_seed(9)).to(cuda_dev)
    base = _logits(ours, ids)
    seen = []

    def hook(mod, hidden, top_k_index, top_k_weights):
        seen.append((mod.layer, tuple(hidden.shape), tuple(top_k_index.shape)))
        return rt.run_layer(mod.layer, hidden, top_k_index, top_k_weights, mod.act_fn)

    rt.capture_hook = hook
    try:
        hooked = _logits(ours, ids)
    finally:
        rt.capture_hook = None
    assert [s[0] for s in seen] == [0, 1]
    assert all(s[1] == (10, 256) and s[2] == (10, 4) for s in seen)
    # same kernels, same inputs: equal up to the fp32 order of the down phase's reductions
    assert float((hooked - base).abs().max() / base.abs().max()) < 1e-3
