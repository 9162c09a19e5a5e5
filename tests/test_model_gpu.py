"""Llama-shaped decode runner (world 1) against an unsharded fp32 PyTorch forward."""
from dataclasses import replace

import pytest
import torch

from comm_opt_b200.models.llama import LlamaWeights, TPDecodeRunner, reference_greedy, tiny_config
from comm_opt_b200.ops.reference import rel_err
from comm_opt_b200.parallel import TPCommunicator

pytestmark = pytest.mark.gpu


def _ref_logits(cfg, full, tokens, device):
    """fp32 logits of the last position of `tokens` [B, T]."""
    import math

    import torch.nn.functional as F

    from comm_opt_b200.ops.reference import rope_tables

    D = cfg.head_dim
    B, P = tokens.shape
    cos, sin = rope_tables(P, D, cfg.rope_theta, device)
    c, sn = cos[None, :, None, :], sin[None, :, None, :]

    def rope(t):
        return torch.cat([t[..., :D // 2] * c - t[..., D // 2:] * sn, t[..., D // 2:] * c + t[..., :D // 2] * sn], -1)

    x = full["embed"].to(device).float()[tokens.to(device).long()]
    for L in full["layers"]:
        L = {k: v.to(device).float() for k, v in L.items()}
        h = F.rms_norm(x, (cfg.hidden,), L["ln1"], cfg.eps)
        qkv = h @ L["wqkv"].t() + (L["bqkv"] if "bqkv" in L else 0.0)
        q, k, v = qkv.split([cfg.heads * D, cfg.kv_heads * D, cfg.kv_heads * D], -1)
        q, k = rope(q.view(B, P, cfg.heads, D)), rope(k.view(B, P, cfg.kv_heads, D))
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2),
                                           v.view(B, P, cfg.kv_heads, D).transpose(1, 2), is_causal=True,
                                           enable_gqa=True, scale=1 / math.sqrt(D))
        x = x + a.transpose(1, 2).reshape(B, P, -1) @ L["wo"].t()
        h = F.rms_norm(x, (cfg.hidden,), L["ln2"], cfg.eps)
        g, u = (h @ L["wgu"].t()).chunk(2, -1)
        x = x + (F.silu(g) * u) @ L["wdown"].t()
    h = F.rms_norm(x[:, -1], (cfg.hidden,), full["final_norm"].to(device).float(), cfg.eps)
    return h @ full["lm_head"].to(device).float().t()


@pytest.mark.parametrize("gemm_impl,model", [("cob", "tiny"), ("torch", "tiny"), ("cob", "tiny-qkv-bias"),
                                             ("cob", "tiny-hd64")])
def test_decode_logits_match_reference(cuda, gemm_impl, model):
    """Decode logits against the fp32 forward; `tiny-qkv-bias` has the Qwen2.5 attention shape (QKV bias,
    5 query heads per KV head)."""
    from comm_opt_b200.models.llama import PRESETS

    cfg = replace(PRESETS[model], layers=2)
    full = LlamaWeights.full_random(cfg, device=cuda, seed=3)
    w = LlamaWeights(cfg, 0, 1, cuda, full=full)
    comm = TPCommunicator(None, device=cuda, dtype=torch.bfloat16, max_rows=8, max_hidden=cfg.hidden)
    runner = TPDecodeRunner(cfg, w, comm, max_batch=4, max_seq=96, device=cuda, gemm=gemm_impl)
    prompts = torch.randint(0, cfg.vocab, (3, 37), generator=torch.Generator().manual_seed(1))
    first = runner.prefill(prompts)
    ref0 = _ref_logits(cfg, full, prompts, cuda)
    assert torch.equal(first.long().cpu(), ref0.argmax(-1).cpu()) or rel_err(
        ref0.gather(1, first.long()[:, None]), ref0.max(-1, keepdim=True).values) < 1e-2
    buf = runner.start(3, first, prompts.shape[1])
    toks = torch.cat([prompts, first.cpu()[:, None].long()], 1)
    for step in range(3):
        runner.step(3, use_graph=False)
        torch.cuda.synchronize()
        ref = _ref_logits(cfg, full, toks, cuda)
        assert rel_err(buf["logits"], ref) < 2 ** -5, (step, rel_err(buf["logits"], ref))
        toks = torch.cat([toks, buf["ids"].cpu()[:, None].long()], 1)
    assert torch.equal(buf["pos"].cpu(), torch.full((3,), 37 + 3, dtype=torch.int32))


def test_graph_replay_equals_eager(cuda):
    cfg = tiny_config(layers=2)
    w = LlamaWeights(cfg, 0, 1, cuda, seed=5)
    comm = TPCommunicator(None, device=cuda, dtype=torch.bfloat16, max_rows=8, max_hidden=cfg.hidden)
    runner = TPDecodeRunner(cfg, w, comm, max_batch=4, max_seq=96, device=cuda)
    prompts = torch.randint(0, cfg.vocab, (4, 20), generator=torch.Generator().manual_seed(2))
    first = runner.prefill(prompts)
    runner.start(4, first, 20)
    eager = []
    for _ in range(4):
        eager.append(runner.step(4, use_graph=False).clone())
    runner.prefill(prompts)
    runner.start(4, first, 20)
    runner.capture(4)
    graph = [runner.step(4).clone() for _ in range(4)]
    torch.cuda.synchronize()
    assert all(torch.equal(a, b) for a, b in zip(eager, graph))
    # qkv, attention, o, norm, down, norm; RoPE + KV append in its own kernel without the fused append; the
    # gate/up projection with its SiLU * up epilogue (one kernel) or the GEMM and the SiLU * up kernel
    per_layer = 6 + (0 if runner.fuse_append else 1) + runner.lin[(0, "gu")].kernels(4)
    assert runner.kernels_per_step[4] == 2 + 2 * per_layer + 2 + 1


def test_smoke_entry(cuda):
    from comm_opt_b200.models.smoke import tiny_decode_step

    out = tiny_decode_step(cuda)
    assert out.shape == (2,)
