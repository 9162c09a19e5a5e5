"""CPU tier for the model description, the fp32 oracles and the analyzers (no GPU, no native code)."""
import json
from dataclasses import replace

import pytest
import torch

from comm_opt_b200.harness.analyze_sweep import calibrate, table
from comm_opt_b200.harness.launch_table import load as load_launches
from comm_opt_b200.harness.launch_table import summarize
from comm_opt_b200.models.llama import LLAMA3_70B, LLAMA3_8B, BlockAllocator, LlamaWeights, tiny_config
from comm_opt_b200.ops.reference import paged_attention_ref, rope_ref, rope_tables
from comm_opt_b200.parallel.communicator import TPCommunicator
from comm_opt_b200.parallel.variant_table import VARIANTS, VariantTable


def test_llama_presets_and_sharding():
    assert abs(LLAMA3_70B.params / 1e9 - 70.6) < 0.2  # Llama-3-70B: 70.6 B parameters
    assert abs(LLAMA3_8B.params / 1e9 - 8.03) < 0.05
    s = LLAMA3_70B.shard(8)
    assert s == dict(nq=8, nkv=1, inter=3584, vocab=16032)
    # the TP=8 decode GEMM shapes the kernels and benches are tuned for
    D = LLAMA3_70B.head_dim
    assert (s["nq"] + 2 * s["nkv"]) * D == 1280 and 2 * s["inter"] == 7168


def test_sharded_weights_slice_the_full_model():
    cfg = tiny_config(layers=1)
    full = LlamaWeights.full_random(cfg, device="cpu", seed=1)
    parts = [LlamaWeights(cfg, r, 2, "cpu", full=full) for r in range(2)]
    # row-parallel o_proj: the ranks' column blocks concatenate to the full matrix
    wo = torch.cat([p.layers[0].wo for p in parts], 1)
    assert torch.equal(wo, full["layers"][0]["wo"])
    # column-parallel gate_up: gate and up halves sharded separately, then stacked per rank
    I = cfg.inter // 2
    g = torch.cat([p.layers[0].wgu[:I] for p in parts], 0)
    assert torch.equal(g, full["layers"][0]["wgu"][:cfg.inter])


def test_block_allocator_reuses_pages():
    a = BlockAllocator(8)
    p1 = a.alloc(5)
    assert len(set(p1)) == 5
    a.release(p1[:3])
    p2 = a.alloc(6)
    assert len(set(p2)) == 6 and not set(p2) & set(p1[3:])


def test_paged_attention_oracle_matches_dense():
    torch.manual_seed(0)
    B, nq, nkv, D, bs, pages = 2, 4, 2, 16, 4, 5
    seq = torch.tensor([7, 17])
    kc = torch.randn(B * pages, nkv, bs, D)
    vc = torch.randn(B * pages, nkv, bs, D)
    bt = torch.randperm(B * pages).view(B, pages).int()
    q = torch.randn(B, nq, D)
    out = paged_attention_ref(q, kc, vc, bt, seq, 0.25)
    for b in range(B):
        k = kc[bt[b].long()].permute(1, 0, 2, 3).reshape(nkv, pages * bs, D)[:, :seq[b]]
        v = vc[bt[b].long()].permute(1, 0, 2, 3).reshape(nkv, pages * bs, D)[:, :seq[b]]
        k, v = k.repeat_interleave(nq // nkv, 0), v.repeat_interleave(nq // nkv, 0)
        ref = torch.softmax(q[b][:, None, :] @ k.transpose(1, 2) * 0.25, -1) @ v
        assert torch.allclose(out[b].float(), ref[:, 0], atol=1e-5)


def test_rope_is_a_rotation():
    cos, sin = rope_tables(64, 32, 1e4)
    x = torch.randn(3, 2, 32)
    pos = torch.tensor([0, 5, 63])
    y = rope_ref(x, pos, cos, sin)
    assert torch.allclose(y[0], x[0].float())                        # position 0: identity
    assert torch.allclose(y.norm(dim=-1), x.float().norm(dim=-1), atol=1e-5)  # norm preserved


def test_interleave_gate_up_roundtrip():
    w = torch.randn(2, 256, 8)
    il = TPCommunicator.interleave_gate_up(w)
    g, u = w[:, :128], w[:, 128:]
    assert torch.equal(il[:, :64], g[:, :64]) and torch.equal(il[:, 64:128], u[:, :64])
    assert torch.equal(il[:, 128:192], g[:, 64:]) and torch.equal(il[:, 192:], u[:, 64:])


def test_launch_table_summary(tmp_path):
    p = tmp_path / "l.csv"
    rows = ['"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"']
    for i, (k, v) in enumerate([("void k_gemm<16>(int)", "10,000"), ("k_attn(x)", "5000"), ("void k_gemm<16>(int)", "10000")]):
        rows.append(f'"{i}","{k}","gpu__time_duration.sum","nsecond","{v}"')
    p.write_text("\n".join(rows) + "\n")
    out = summarize(load_launches(str(p)), steps=1)
    assert out[0][0].startswith("void k_gemm") and out[0][1] == 2 and abs(out[0][2] - 20.0) < 1e-9
    assert abs(sum(r[3] for r in out) - 1.0) < 1e-9


def test_analyze_and_calibrate_synthetic_sweep(tmp_path):
    rows = []
    for T, (a1, a2, b) in {1: (5.0, 9.0, 10.0), 64: (20.0, 12.0, 30.0)}.items():
        for impl, us in (("ours:lamport_1s", a1), ("ours:lamport_2s", a2), ("vllm_car", b)):
            rows.append(dict(impl=impl, world=8, dtype="bfloat16", hidden=8192, tokens=T, bytes=T * 16384,
                             p50_us=us, correct=True, skip="", variant=dict(blocks=8, threads=128, cluster=1)))
    text, summary = table(rows)
    assert "speedup" in text and len(summary) == 2
    t = calibrate(rows, tmp_path / "vt.json")
    c1 = t.lookup(8, torch.bfloat16, 2, 8192, 1, False)
    c64 = t.lookup(8, torch.bfloat16, 2, 8192, 64, False)
    assert c1.variant == VARIANTS["lamport_1s"] and c64.variant == VARIANTS["lamport_2s"]
    t.save(tmp_path / "vt.json")
    again = VariantTable.load(tmp_path / "vt.json")
    assert again.lookup(8, torch.bfloat16, 2, 8192, 64, False).variant == VARIANTS["lamport_2s"]
    json.loads((tmp_path / "vt.json").read_text())
    # NVLink roofline at a given link rate: 2 (W - 1) / W x 1 MB at 770 GB/s = 2.38 us; fastest of ours at 64 tokens is 12 us
    from comm_opt_b200.harness.analyze_sweep import roofline_table

    text, summ = roofline_table(rows, link_gbs=770.0)
    r64 = next(r for r in summ if r["tokens"] == 64)
    assert r64["ours"] == "ours:lamport_2s" and abs(r64["target_us"] - 2.383) < 1e-2
    assert abs(r64["fraction"] - r64["target_us"] / 12.0) < 1e-9 and r64["baseline"] == "vllm_car"


def test_attention_split_plans():
    """Split-KV geometry: covers every page, at most 512 pages per split (the kernel's page list),
    one wave of resident CTAs, cluster merge for 2..16 splits, 16 only for long contexts."""
    from comm_opt_b200.ops.kernels import ATTN_CTAS_PER_SM, attention_split_plan

    for batch in (1, 2, 8, 32, 128):
        for nkv in (1, 2, 8):
            for pages in (1, 7, 64, 136, 512, 2048):
                splits, pps, cluster = attention_split_plan(batch, nkv, pages, 148)
                assert splits >= 1 and 1 <= pps <= 512 and splits * pps >= pages and (splits - 1) * pps < pages
                assert cluster == (1 < splits <= 16)
                if splits > 1:
                    assert batch * nkv * splits <= ATTN_CTAS_PER_SM * 148 or pps == 512
                if splits > 8 and pps < 512:
                    assert (pages + 7) // 8 > 32  # 16-way clusters only where 8 splits keep > 32 pages
    assert attention_split_plan(8, 1, 128, 148) == (8, 16, True)  # 70B TP=8, 2048 tokens
    assert attention_split_plan(8, 1, 512, 148) == (16, 32, True)  # 8192 tokens: a 16-CTA cluster
    assert attention_split_plan(32, 1, 512, 148)[2] and attention_split_plan(32, 1, 512, 148)[0] == 8


def test_repeat_statistics_effectiveness_rule():
    from comm_opt_b200.harness.analyze_sweep import repeats

    rows = []
    for rep, (a, b) in enumerate([(10.0, 12.0), (10.2, 12.5), (10.1, 12.2)]):
        for impl, v in (("ours:x", a), ("base", b)):
            rows.append(dict(world=8, tokens=1, impl=impl, p50_us=v, correct=True))
            rows.append(dict(world=8, tokens=2, impl=impl, p50_us=v + (rep == 0) * 3.0, correct=True))
    out = {r["tokens"]: r for r in repeats(rows, "ours:x", "base")}
    assert out[1]["effective"] and abs(out[1]["ours"]["med"] - 10.1) < 1e-9 and out[1]["ours"]["n"] == 3
    assert not out[2]["effective"]  # the first launch's outlier makes the intervals overlap


def test_qwen25_32b_preset_and_bias_sharding():
    """Qwen2.5-32B shapes (the reference's end-to-end inference model, hidden 5120): 32.8 B parameters,
    5 query heads per KV head at TP=8, and the QKV bias sharded with the same q / k / v head split as
    the weight rows."""
    from comm_opt_b200.models.llama import PRESETS, QWEN25_32B

    assert abs(QWEN25_32B.params / 1e9 - 32.76) < 0.05
    for tp in (1, 2, 4, 8):
        s = QWEN25_32B.shard(tp)
        assert s["nq"] // s["nkv"] == 5 and s["nq"] * tp == 40
    s = QWEN25_32B.shard(8)
    assert s == dict(nq=5, nkv=1, inter=3456, vocab=19008)
    cfg = PRESETS["tiny-qkv-bias"]
    full = LlamaWeights.full_random(cfg, device="cpu", seed=2)
    assert all("bqkv" in L for L in full["layers"])
    assert all("bqkv" not in L for L in LlamaWeights.full_random(tiny_config(layers=1), device="cpu")["layers"])
    tp, D = 2, cfg.head_dim
    parts = [LlamaWeights(cfg, r, tp, "cpu", full=full) for r in range(tp)]
    b = full["layers"][0]["bqkv"]
    w = full["layers"][0]["wqkv"]
    nq, nkv = cfg.heads // tp, cfg.kv_heads // tp
    for r, p in enumerate(parts):
        L = p.layers[0]
        assert L.bqkv.shape == ((nq + 2 * nkv) * D,)
        q0, k0, v0 = r * nq * D, cfg.heads * D + r * nkv * D, (cfg.heads + cfg.kv_heads) * D + r * nkv * D
        assert torch.equal(L.bqkv[:nq * D], b[q0:q0 + nq * D])
        assert torch.equal(L.bqkv[nq * D:(nq + nkv) * D], b[k0:k0 + nkv * D])
        assert torch.equal(L.bqkv[(nq + nkv) * D:], b[v0:v0 + nkv * D])
        assert torch.equal(L.wqkv[nq * D:(nq + nkv) * D], w[k0:k0 + nkv * D])  # weight rows split alike
    # random-init (unsliced) shards carry a bias of the right length too
    own = LlamaWeights(cfg, 1, tp, "cpu", seed=4)
    assert own.layers[0].bqkv.shape == ((nq + 2 * nkv) * D,)


def test_tinyllama_kv_head_replication():
    """TinyLlama-1.1B (the reference's small end-to-end model): at TP = 8 its 4 KV heads are replicated
    on 2 ranks each; ranks that share a KV head hold the same k / v rows, and its query heads are the
    ones that attend to that head."""
    from comm_opt_b200.models.llama import PRESETS, TINYLLAMA

    assert abs(TINYLLAMA.params / 1e9 - 1.10) < 0.01
    assert TINYLLAMA.shard(8) == dict(nq=4, nkv=1, inter=704, vocab=4000)
    assert [TINYLLAMA.kv_head0(r, 8) for r in range(8)] == [0, 0, 1, 1, 2, 2, 3, 3]
    assert [TINYLLAMA.kv_head0(r, 2) for r in range(2)] == [0, 2]
    cfg = replace(PRESETS["tiny-hd64"], layers=1)
    full = LlamaWeights.full_random(cfg, device="cpu", seed=3)
    tp, D = 4, cfg.head_dim
    parts = [LlamaWeights(cfg, r, tp, "cpu", full=full) for r in range(tp)]
    w = full["layers"][0]["wqkv"]
    k_full = w[cfg.heads * D:(cfg.heads + cfg.kv_heads) * D]
    for r, p in enumerate(parts):
        wq = p.layers[0].wqkv
        assert wq.shape[0] == (cfg.heads // tp + 2) * D
        kv = cfg.kv_head0(r, tp)
        assert kv * (cfg.heads // cfg.kv_heads) <= r * (cfg.heads // tp) < (kv + 1) * (cfg.heads // cfg.kv_heads)
        assert torch.equal(wq[cfg.heads // tp * D:(cfg.heads // tp + 1) * D], k_full[kv * D:(kv + 1) * D])
    assert torch.equal(parts[0].layers[0].wqkv[4 * D:], parts[1].layers[0].wqkv[4 * D:])
    # random-init shards: replicas of one KV head get the same k / v rows, different q rows
    own = [LlamaWeights(cfg, r, tp, "cpu", seed=5) for r in (0, 1, 2)]
    q = cfg.heads // tp * D
    assert torch.equal(own[0].layers[0].wqkv[q:], own[1].layers[0].wqkv[q:])
    assert not torch.equal(own[0].layers[0].wqkv[q:], own[2].layers[0].wqkv[q:])
    assert not torch.equal(own[0].layers[0].wqkv[:q], own[1].layers[0].wqkv[:q])


class _GateUpRec:
    """Recorder for the runner's gate/up projection (GateUpLinear): one GEMM with the SwiGLU epilogue
    (`fused`), or the GEMM and the SiLU * up kernel."""

    def __init__(self, calls, fused=False, inputs=None, key=None):
        self.calls, self.fused, self.inputs, self.key = calls, fused, inputs, key

    def kernels(self, M):
        return 1 if self.fused else 2

    def __call__(self, x, out=None):
        if self.inputs is not None:
            self.inputs.append((self.key, x))
        self.calls += ["gemm:swiglu"] if self.fused else ["gemm", "silu_mul"]


def _recording_runner(monkeypatch, layers, tp, fuse, kinds, epi, gu_fused=False):
    """A TPDecodeRunner whose kernels, GEMMs and collective are recorders (no GPU): the decode step's
    composition and its kernel count can be checked on CPU."""
    from types import SimpleNamespace

    import comm_opt_b200.models.llama as M

    calls = []

    class Rec:
        def __getattr__(self, name):
            return lambda *a, **k: calls.append(name)

    class Comm:
        def gemm_push(self, *a, **k):
            calls.append("gemm_push")

        def ar_norm_gemm(self, *a, epilogue=None, **k):
            calls.append("ar_norm_gemm" + (f":{epilogue}" if epilogue else ""))

        def fused_allreduce_add_rmsnorm(self, *a, **k):
            calls.append("fused_ar")

        def all_gather_u32(self, *a, **k):
            calls.append("all_gather")

    monkeypatch.setattr(M, "K", Rec())
    cfg = replace(M.TINY, layers=layers)
    r = object.__new__(M.TPDecodeRunner)
    r.cfg, r.s, r.tp, r.rank = cfg, cfg.shard(tp), tp, 0
    r.w = M.LlamaWeights(cfg, 0, tp, "cpu", seed=1)
    r.comm, r.collective, r.nccl_group, r.gemm = Comm(), "ours", None, "cob"
    r._car = r._vllm_ops = None
    keys = [(i, n) for i in range(layers) for n in ("qkv", "o", "gu", "down")] + ["head"]
    r.lin = {k: (_GateUpRec(calls, gu_fused) if k[1:] == ("gu",) else (lambda *a, **kw: calls.append("gemm")))
             for k in keys}
    r.cache = SimpleNamespace(block_tables=torch.zeros(4, 8, dtype=torch.int32), k=[None] * layers, v=[None] * layers)
    r.cos = r.sin = None
    r.scale = 1.0
    r.fuse_boundary, r.fuse_kinds, r.fuse_epilogues = fuse, {4: kinds}, any(epi)
    r._fuse_epi, r._wgu_il, r.epi_use = {4: epi}, [None] * layers, {}
    r.fuse_append = False
    buf = {k: torch.zeros(4, 8) for k in ("ids", "pos", "lens", "res", "h", "part", "qkv", "q", "attn", "gu", "act",
                                           "logits")}
    buf["keys"] = torch.zeros(4, dtype=torch.int64)
    buf["gathered"] = torch.zeros(tp, 4, dtype=torch.int64)
    buf["attn_op"] = lambda *a, **k: calls.append("attention")
    return r, buf, calls


def _expected_step(layers, fuse, kinds, epi, append=False, gu_fused=False):
    seq = _expected_step_kernels(layers, fuse, kinds, epi, gu_fused)
    # the fused append folds every RoPE + KV append kernel into the attention kernel that follows it
    return [k for k in seq if k != "rope_append_kv"] if append else seq


def _expected_step_kernels(layers, fuse, kinds, epi, gu_fused=False):
    fa, fm = kinds if fuse else (False, False)
    sw, rp = (epi[0] and fa, epi[1] and fm) if fuse else (False, False)
    gu = ["gemm:swiglu"] if gu_fused else ["gemm", "silu_mul"]  # the separate gate/up projection
    seq = ["embedding", "rmsnorm", "gemm"]
    for i in range(layers):
        last = i + 1 == layers
        if i == 0 or not rp:
            seq.append("rope_append_kv")
        seq.append("attention")
        if fa:
            seq += ["gemm_push", "ar_norm_gemm:swiglu"] if sw else ["gemm_push", "ar_norm_gemm", "silu_mul"]
        else:
            seq += ["gemm", "fused_ar"] + gu
        if fm:
            seq += ["gemm_push", "ar_norm_gemm:rope_kv" if rp and not last else "ar_norm_gemm"]
        else:
            seq += ["gemm", "fused_ar", "gemm"]
    if not fuse:  # the separate step issues the next layer's QKV GEMM at the top of the layer
        seq = ["embedding", "rmsnorm"]
        for i in range(layers):
            seq += ["gemm", "rope_append_kv", "attention", "gemm", "fused_ar"] + gu + ["gemm", "fused_ar"]
        seq.append("gemm")
    return seq + ["argmax_local", "all_gather", "argmax_combine"]


def test_decode_step_composition_every_boundary_mix(monkeypatch):
    """Every mix of fused / separate layer boundaries (and the GEMM epilogues) issues the expected
    kernel sequence, and the step's kernel count (the bench's `gpu_launches`) matches it."""
    import itertools

    for fuse in (True, False):
        for kinds in itertools.product((True, False), repeat=2):
            for epi in itertools.product((False, True), repeat=2):
                for append in (False, True):
                    for gf in (False, True):
                        r, buf, calls = _recording_runner(monkeypatch, 3, 2, fuse, kinds, epi, gu_fused=gf)
                        r.fuse_append = append
                        n = r._step(4, buf)
                        case = (fuse, kinds, epi, append, gf)
                        assert calls == _expected_step(3, fuse, kinds, epi, append, gf), case
                        assert n == len(calls), (case, n, len(calls))


def test_decode_step_composition_vllm_stack(monkeypatch):
    """The reference's baseline stack in the same step: vLLM custom all-reduce (out of place) + vLLM
    fused_add_rms_norm at both boundaries, the next GEMM reading the all-reduce's output; the kernel count
    names only this package's kernels."""
    from types import SimpleNamespace

    r, buf, calls = _recording_runner(monkeypatch, 2, 2, False, (False, False), (False, False))
    seen = {}

    def car_ar(x):
        calls.append("car_ar")
        seen["out"] = torch.zeros_like(x)
        return seen["out"]

    r.collective = "vllm"
    r._car = SimpleNamespace(custom_all_reduce=car_ar)
    r._vllm_ops = SimpleNamespace(fused_add_rms_norm=lambda out, res, g, eps: calls.append("vllm_norm"))
    gemm_inputs = []
    for k in list(r.lin):
        r.lin[k] = (_GateUpRec(calls, False, gemm_inputs, k) if k[1:] == ("gu",) else
                    (lambda x, out=None, _k=k: (gemm_inputs.append((_k, x)), calls.append("gemm"))))
    n = r._step(4, buf)
    layer = ["gemm", "rope_append_kv", "attention", "gemm", "car_ar", "vllm_norm", "gemm", "silu_mul", "gemm",
             "car_ar", "vllm_norm"]
    assert calls == ["embedding", "rmsnorm"] + layer * 2 + ["gemm", "argmax_local", "all_gather", "argmax_combine"]
    assert n == len(calls) - 4 * 2  # two vLLM kernels at each of the two boundaries of both layers
    # the GEMM after a boundary reads the all-reduce's output, not buf["h"]
    gu = [x for k, x in gemm_inputs if k == (1, "gu")][0]
    assert gu is not buf["h"] and [x for k, x in gemm_inputs if k == "head"][0] is seen["out"]


def test_pack_weight_layout_and_round_trip():
    """Packed decode-GEMM weights: 128 x 64 blocks in (tile, k-step) order, 16-byte chunk c of row r at
    chunk position c ^ (r % 8), rows past N zero; dense() restores the row-major weight."""
    from comm_opt_b200.models.gemm import pack_weight

    for N, K in [(128, 64), (300, 192), (1280, 1024)]:
        w = torch.randn(N, K).bfloat16()
        p = pack_weight(w)
        assert p.shape == (N, K) and p.data.shape == ((N + 127) // 128, K // 64, 128, 64)
        assert torch.equal(p.dense(), w)
        blocks = p.data.view(p.data.shape[0], K // 64, 128, 8, 8)
        for t in range(blocks.shape[0]):
            for ks in range(K // 64):
                for r in (0, 5, 77, 127):
                    for c in range(8):
                        n = t * 128 + r
                        got = blocks[t, ks, r, c ^ (r & 7)]
                        want = w[n, ks * 64 + c * 8: ks * 64 + c * 8 + 8] if n < N else torch.zeros(8).bfloat16()
                        assert torch.equal(got, want)
    with pytest.raises(ValueError):
        pack_weight(torch.zeros(128, 100))


def test_gate_up_interleave_round_trip_and_split_rule():
    """Gate/up rows interleaved by 64 for the SwiGLU epilogue: every 128-row tile holds 64 gate rows and
    their up rows; packing with the interleave keeps dense() the original [gate; up] weight; the split
    counts the epilogue accepts are the launched ones that divide 64."""
    from comm_opt_b200.models.gemm import (candidates, cluster_split_count, deinterleave_rows, interleave_rows,
                                           pack_weight, swiglu_splits)

    I, K = 192, 128
    w = torch.randn(2 * I, K).bfloat16()
    wi = interleave_rows(w, 64)
    for t in range(I // 64):
        assert torch.equal(wi[128 * t:128 * t + 64], w[64 * t:64 * t + 64])
        assert torch.equal(wi[128 * t + 64:128 * t + 128], w[I + 64 * t:I + 64 * t + 64])
    assert torch.equal(deinterleave_rows(wi, 64), w)
    p = pack_weight(w, interleave=64)
    assert p.il == 64 and torch.equal(p.dense(), w) and torch.equal(pack_weight(wi).data, p.data)
    w3 = torch.randn(2, 2 * I, K).bfloat16()  # emulated ranks
    assert torch.equal(pack_weight(w3, interleave=64).dense(), w3)
    with pytest.raises(ValueError):
        interleave_rows(torch.zeros(2 * 96, 64), 64)
    assert cluster_split_count(8192, 16) == 16 and cluster_split_count(512, 16) == 8
    assert cluster_split_count(1024, 3) == 3 and cluster_split_count(1024, 6) == 6
    assert [s for s in (2, 3, 4, 6, 8, 12, 16) if swiglu_splits(8192, s)] == [2, 4, 8, 16]
    assert not swiglu_splits(64, 2)  # one k-step: one CTA per tile
    c = candidates(8, 7168, 8192, 148, swiglu=True)
    assert c and all(x.get("swiglu") and (not x.get("cluster_splits") or swiglu_splits(8192, x["cluster_splits"]))
                     for x in c)
    assert {"small_smem": True, "swiglu": True} in c and {"swiglu": True} in c  # stream-K at M <= 16
    assert all(x.get("cluster_splits") for x in candidates(32, 7168, 8192, 148, swiglu=True))


def test_variant_table_validation_rule():
    """Fresh launches of ours:auto against fixed variants: within 3 %, or retuned only when a variant is
    >= 3 % faster with disjoint [min, max] intervals over >= 3 launches."""
    from comm_opt_b200.harness.analyze_sweep import validate

    def rows(auto, fixed, T):
        out = []
        for a, f in zip(auto, fixed):
            out.append(dict(world=8, dtype="bfloat16", hidden=8192, tokens=T, impl="ours:auto", p50_us=a, correct=True))
            out.append(dict(world=8, dtype="bfloat16", hidden=8192, tokens=T, impl="ours:lamport_2s", p50_us=f,
                            correct=True))
        return out

    res = {r["tokens"]: r for r in validate(rows([10.0, 10.1, 10.2], [9.9, 10.0, 10.3], 8) +
                                            rows([12.0, 12.2, 12.1], [10.0, 10.1, 10.2], 64) +
                                            rows([12.0, 9.0, 12.1], [10.0, 10.1, 10.2], 128))}
    assert res[8]["within"] and not res[8]["retune"]
    assert not res[64]["within"] and res[64]["retune"] and res[64]["best"] == "ours:lamport_2s"
    assert not res[128]["retune"]  # 18 % slower by the median, but the intervals overlap


def test_gate_up_linear_keeps_the_faster_form(monkeypatch):
    """GateUpLinear.tune: the SwiGLU-epilogue launch is kept only when it measures no slower than the best
    plain launch plus the SiLU * up kernel; weights not interleaved by 64 (or cuBLAS) never use it."""
    import comm_opt_b200.models.gemm as G

    w = G.pack_weight(torch.zeros(256, 128).bfloat16(), interleave=64)
    times = {}

    def fake_tune(weight, M, iters=20, swiglu=False):
        return dict(times["sw" if swiglu else "plain"], us=times["sw_us" if swiglu else "plain_us"])

    monkeypatch.setattr(G, "tune", fake_tune)
    monkeypatch.setattr(G, "_silu_us", lambda M, inter, dtype, device: 2.0)
    for sw_us, plain_us, fused in ((143.0, 141.5, True), (144.0, 141.5, False), (20.8, 20.5, True)):
        times.update(sw=dict(cluster_splits=4, small_smem=True, swiglu=True), plain=dict(small_smem=True),
                     sw_us=sw_us, plain_us=plain_us)
        lin = G.GateUpLinear(w)
        lin.tune(8)
        assert (lin.kernels(8) == 1) == fused, (sw_us, plain_us)
        assert (lin.fused[8] == times["sw"]) if fused else (lin.cfg[8] == {"small_smem": True})
    plain_w = G.pack_weight(torch.zeros(256, 128).bfloat16())  # [gate; up] rows: no epilogue
    lin = G.GateUpLinear(plain_w)
    lin.tune(8)
    assert lin.kernels(8) == 2 and lin.il == 0
    lin = G.GateUpLinear(torch.zeros(256, 128).bfloat16(), impl="torch")
    lin.tune(8)
    assert lin.kernels(8) == 2
