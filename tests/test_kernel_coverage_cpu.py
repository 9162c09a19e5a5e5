"""Work partitioning of the fused all-reduce kernels, restated on CPU (no GPU).

For every geometry the host launcher accepts (resolve_config through `fused_ar_config`), the index
arithmetic of csrc/fused_ar.cu is replayed thread by thread in Python and every (row, 16-byte vector)
of the message must be handled exactly once in each phase, with every index inside the heap layout.
This checks the thread/vector mapping (the one-vector one-shot form chosen at launch, the two-shot
units and flat phases, the multicast two-shot's last phase in row groups of 32) without running a
kernel.
"""
import numpy as np
import pytest

from comm_opt_b200._ext import available

pytestmark = pytest.mark.skipif(not available(), reason="native extension not built")

EPV = {0: 4, 1: 8, 2: 8}  # elements per 16-byte vector by dtype code (f32, f16, bf16)
KVPT = 4


def _config(world, rows, hidden, dtype, variant, emulate=0, sms=148, blocks=0, threads=0, cluster=0):
    from comm_opt_b200._ext import native

    C = native()
    esz = 4 if dtype == 0 else 2
    L = C.plan_layout(world, 512, 8192, esz, 4096)
    rc, v, b, t, cl = C.fused_ar_config(L, world, rows, hidden, dtype, variant, blocks, threads, cluster, emulate,
                                        sms, True)
    return rc, b, t, cl, L


def oneshot_cover(rows, hv, blocks, threads, cluster):
    """k_oneshot: cluster cl = b // C owns rows cl, cl + ncl, ...; CTA crank = b % C owns the vector chunk
    [crank * chunk, ...); thread tid handles v0 + tid + k * NT for k < VPT (VPT = 1 when the chunk fits)."""
    C = cluster
    chunk = (hv + C - 1) // C
    vpt = 1 if chunk <= threads else KVPT
    seen = np.zeros((rows, hv), dtype=np.int32)
    ncl = blocks // C
    tid = np.arange(threads)
    for b in range(blocks):
        crank, cl = b % C, b // C
        v0, v1 = crank * chunk, min(hv, crank * chunk + chunk)
        for row in range(cl, rows, ncl):
            for k in range(vpt):
                v = v0 + tid + k * threads
                v = v[v < v1]
                np.add.at(seen[row], v, 1)
    return seen


def twoshot_phase2_units(rows, hv, world, blocks, threads, variant):
    """k_twoshot phase 2: units of 32 vectors of each rank's owned column slice; LAMPORT spreads
    (row, unit) over all warps of the grid, PULL / NVLS keep a row in the block that staged it. Returns
    how often each (row, owned vector) is reduced by one rank."""
    sv = hv // world
    U = (sv + 31) // 32
    nw = threads // 32
    seen = np.zeros((rows, sv), dtype=np.int32)
    if variant == 2:  # LAMPORT: flat over grid warps
        total_warps = blocks * nw
        for gw in range(total_warps):
            for g in range(gw, rows * U, total_warps):
                row, c0 = g // U, (g % U) * 32
                i = c0 + np.arange(32)
                np.add.at(seen[row], i[i < sv], 1)
    else:
        for b in range(blocks):
            nunits = ((rows - b + blocks - 1) // blocks) * U
            if variant == 4:  # NVLS: kNvB = 4 units per warp and step
                for warp in range(nw):
                    for g0 in range(warp, nunits, nw * 4):
                        for j in range(4):
                            g = g0 + j * nw
                            if g < nunits:
                                row, c0 = b + (g // U) * blocks, (g % U) * 32
                                i = c0 + np.arange(32)
                                np.add.at(seen[row], i[i < sv], 1)
            else:
                for warp in range(nw):
                    for g in range(warp, nunits, nw):
                        row, c0 = b + (g // U) * blocks, (g % U) * 32
                        i = c0 + np.arange(32)
                        np.add.at(seen[row], i[i < sv], 1)
    return seen


def twoshot_phase3(rows, hv, blocks, threads, variant):
    """k_twoshot phase 3: LAMPORT / PULL flat over (row, v), two vectors per lane per step (a warp shares
    one row per step); NVLS: the block's rows in groups of 32, every thread four vectors per step."""
    seen = np.zeros((rows, hv), dtype=np.int32)
    if variant != 4:
        total, gthreads = rows * hv, blocks * threads
        for gtid0 in range(0, gthreads, 32):  # warps: u0 = gtid - lane
            for u0 in range(gtid0, total, 2 * gthreads):
                for k in range(2):
                    ub = u0 + k * gthreads
                    if ub < total:
                        row = ub // hv
                        v = ub + np.arange(32) - row * hv
                        assert (v < hv).all(), "a warp's 32 vectors stay in one row (hv % 32 == 0)"
                        np.add.at(seen[row], v, 1)
    else:
        for b in range(blocks):
            nrows_b = (rows - b + blocks - 1) // blocks
            for r0 in range(0, nrows_b, 32):
                nr = min(32, nrows_b - r0)
                items = nr * hv
                tid = np.arange(threads)
                for i0 in range(0, items, 4 * threads):
                    for k in range(4):
                        idx = i0 + tid + k * threads
                        idx = idx[idx < items]
                        rl, v = idx // hv, idx % hv
                        for r, vv in zip(rl, v):
                            seen[b + (r0 + r) * blocks, vv] += 1
    return seen


SHAPES = [(1, 8192), (3, 5120), (8, 8192), (17, 2048), (64, 4096), (128, 8192)]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("variant", [1, 3, 5, 7])
def test_oneshot_covers_every_vector_once(world, variant):
    for rows, hidden in SHAPES:
        for emulate in (0, 1):
            rc, b, t, cl, L = _config(world, rows, hidden, 2, variant, emulate)
            assert rc == 0, (world, variant, rows, hidden)
            hv = hidden // EPV[2]
            seen = oneshot_cover(rows, hv, b, t, cl)
            assert (seen == 1).all(), (world, variant, rows, hidden, b, t, cl)
    # explicit clusters and block counts, as the calibrated table and the tests use them
    for cluster in (1, 2, 4, 8):
        rc, b, t, cl, L = _config(world, 4, 8192, 2, variant, blocks=4 * cluster, cluster=cluster)
        assert rc == 0
        assert (oneshot_cover(4, 1024, b, t, cl) == 1).all()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("variant", [2, 4, 6])
def test_twoshot_phases_cover_every_vector_once(world, variant):
    for rows, hidden in SHAPES:
        rc, b, t, cl, L = _config(world, rows, hidden, 2, variant)
        hv = hidden // EPV[2]
        if hv % world or hv % 32:
            assert rc != 0
            continue
        assert rc == 0 and cl == 1 and b <= 148
        p2 = twoshot_phase2_units(rows, hv, world, b, t, variant)
        assert (p2 == 1).all(), ("phase 2", world, variant, rows, hidden, b, t)
        p3 = twoshot_phase3(rows, hv, b, t, variant)
        assert (p3 == 1).all(), ("phase 3", world, variant, rows, hidden, b, t)
    # more CTAs than rows (the pull two-shot's default for small messages, and explicit grids)
    for blocks in (1, 3, 16, 40):
        rc, b, t, cl, L = _config(world, 4, 8192, 2, variant, blocks=blocks, threads=256)
        if rc != 0:
            continue
        assert (twoshot_phase2_units(4, 1024, world, b, t, variant) == 1).all()
        assert (twoshot_phase3(4, 1024, b, t, variant) == 1).all()


def test_pull_twoshot_default_grid_has_gather_ctas():
    """The pull two-shot now starts enough CTAs for its flat gather phase even for one row."""
    rc, b, t, cl, L = _config(8, 1, 8192, 2, 6)
    assert rc == 0 and b == 1024 // t
    rc, b, t, cl, L = _config(8, 8, 8192, 2, 6)
    assert rc == 0 and b == 8 * 1024 // t


def test_attention_pages_and_merge_cover_once():
    """k_decode_attn: the sequence's pages are cut by its actual length into `splits` parts of
    min(pps, ceil(npages / splits)) pages; split s reads page-table entries [pg0, pg1) (inside the row)
    and attends them with warp w taking pg0 + w, pg0 + w + 4, ...; the cluster merge gives CTA r output
    elements [r * per, (r + 1) * per). Every page of every sequence is attended once, no split holds more
    than the plan's pps pages, and every output element is written once, for the split plans of the
    decode shapes."""
    from comm_opt_b200.ops.kernels import attention_split_plan

    kWarps, kBS = 4, 16
    for batch, nkv, G, D in [(8, 1, 8, 128), (8, 8, 8, 128), (1, 1, 8, 128), (32, 1, 5, 128), (8, 1, 4, 64)]:
        for max_pages in (1, 7, 33, 129, 513):
            splits, pps, cluster = attention_split_plan(batch, nkv, max_pages, 148)
            for seq in {x for x in (1, 15, 16, 17, max_pages * kBS // 2 + 3, max_pages * kBS) if x <= max_pages * kBS}:
                npages = (seq + kBS - 1) // kBS
                seen = np.zeros(npages, dtype=np.int32)
                dyn = min(pps, max(1, -(-npages // splits)))
                for split in range(splits):
                    pg0 = split * dyn
                    pg1 = min(npages, pg0 + dyn)
                    assert pg1 <= max_pages  # table reads stay inside the row
                    for warp in range(kWarps):
                        my = (pg1 - pg0 - warp + kWarps - 1) // kWarps if pg1 - pg0 > warp else 0
                        assert my <= pps
                        for i in range(my):
                            seen[pg0 + warp + i * kWarps] += 1
                assert (seen == 1).all(), (batch, nkv, max_pages, seq, splits, pps)
            if cluster:
                per = (G * D + splits - 1) // splits
                out = np.zeros(G * D, dtype=np.int32)
                for r in range(splits):
                    out[r * per:min(G * D, (r + 1) * per)] += 1
                assert (out == 1).all()


def test_layer_boundary_pieces_and_push_groups_cover_once():
    """Layer-boundary GEMMs (csrc/fused_gemm.cu) for every decode projection of the model presets at
    TP 2/4/8: the consumer's pieces (CTA (t, r) reduces vectors [vb, ve) of split r's k-range) cover the
    K vectors of every row exactly once, and the push epilogue's feature groups (split r of tile t
    pushes features [r * BM / cs, (r + 1) * BM / cs)) cover every output feature exactly once."""
    from comm_opt_b200._ext import native
    from comm_opt_b200.models.llama import PRESETS

    C = native()
    BM, BK = 128, 64
    for model in ("70b", "8b", "qwen2.5-32b", "tinyllama-1.1b"):
        cfg = PRESETS[model]
        for tp in (2, 4, 8):
            s, D, H = cfg.shard(tp), cfg.head_dim, cfg.hidden
            consumers = [((s["nq"] + 2 * s["nkv"]) * D, H), (2 * s["inter"], H), (s["vocab"], H)]
            pushes = [(H, s["nq"] * D), (H, s["inter"])]
            for M in (1, 8, 32, 128):
                for N, K in consumers:
                    bn, tiles, splits, kps, xctas, ctas, smem = C.fused_gemm_plan(M, N, K, 0, 148, True, 0)
                    if splits == 0:
                        continue
                    KT, KV = K // BK, K // 8
                    assert splits * kps >= KT and ctas <= min(148 * (2 if bn <= 64 else 1), 296)
                    seen = np.zeros(KV, dtype=np.int32)
                    for r in range(splits):
                        k0 = r * kps
                        s0, slen = k0 * 8, min(KV, (k0 + kps) * 8) - k0 * 8
                        for t in range(xctas):
                            vb, ve = s0 + slen * t // xctas, s0 + slen * (t + 1) // xctas
                            seen[vb:ve] += 1
                    assert (seen == 1).all(), (model, tp, M, N, K, splits, kps, xctas)
                for N, K in pushes:
                    bn, tiles, splits, kps, xctas, ctas, smem = C.fused_gemm_plan(M, N, K, 0, 148, False, 0)
                    assert splits >= 1 and BM % (8 * splits) == 0 and splits * kps >= K // BK
                    per = BM // splits
                    feats = np.zeros(tiles * BM, dtype=np.int32)
                    for t in range(tiles):
                        for r in range(splits):
                            feats[t * BM + r * per:t * BM + (r + 1) * per] += 1
                    assert (feats[:N] == 1).all(), (model, tp, M, N, K, splits)


def test_attention_shared_memory_keeps_two_ctas_per_sm():
    """The split planner assumes two resident attention CTAs per SM (ATTN_CTAS_PER_SM): with the shallow KV
    ring every launch form - no merge, the push merge of 2..8-CTA clusters (its buffer grows with the
    query group and the split count), the pull merge of 9..16 - fits twice into one SM's 228 KB (each
    CTA also holds 1 KB for the driver); the deep ring fits one CTA per SM (227 KB per block)."""
    from comm_opt_b200._ext import native
    from comm_opt_b200.ops.kernels import ATTN_CTAS_PER_SM

    C = native()
    sm_bytes, block_max = 228 * 1024, 227 * 1024
    for D in (64, 128):
        for group in range(1, 17):
            for splits in range(1, 17):
                for cluster in (False, True):
                    shallow = C.attn_launch_smem_bytes(splits, group, D, cluster, 3)
                    assert ATTN_CTAS_PER_SM * (shallow + 1024) <= sm_bytes, (D, group, splits, cluster, shallow)
                    deep = C.attn_launch_smem_bytes(splits, group, D, cluster, 6)
                    assert deep + 1024 <= block_max, (D, group, splits, cluster, deep)
                    if cluster and 1 < splits <= 8:  # the push merge's buffer: partials + (max, sum) rows
                        per = -(-group * D // splits)
                        assert shallow - C.attn_launch_smem_bytes(splits, group, D, False, 3) == \
                            4 * (splits * per + splits * group * 2)


def test_attention_push_merge_slots():
    """k_decode_attn's push merge (clusters of 2..8): split s stores its partial of output element idx at
    slot s * per + (idx - o * per) of owner o = idx // per and its (max, sum) of row g at (s * G + g) * 2
    of every CTA; owner r folds, for each of its elements, slot c * per + (idx - r * per) of every split c.
    Every owner slot is written exactly once, stays inside the buffer that attn_push_bytes sizes, and
    holds exactly the partial the owner reads for that (split, element)."""
    for G in (1, 4, 5, 8, 16):
        for D in (64, 128):
            for cs in range(2, 9):
                per = -(-G * D // cs)
                written = {}
                for s in range(cs):
                    for idx in range(G * D):
                        o = idx // per
                        key = (o, s * per + (idx - o * per))
                        assert key not in written and key[1] < cs * per
                        written[key] = (s, idx)
                    for c in range(cs):
                        for g in range(G):
                            assert (s * G + g) * 2 + 1 < cs * G * 2
                for r in range(cs):
                    for idx in range(r * per, min(G * D, (r + 1) * per)):
                        for c in range(cs):
                            assert written[(r, c * per + (idx - r * per))] == (c, idx)
                assert len(written) == cs * G * D


def test_gemm_swiglu_row_pairing():
    """Decode GEMM SwiGLU epilogue, gate/up rows interleaved by 64 in a 128-row tile. Cluster form (s CTAs,
    s | 64): row `row` goes to owner f // ph, slot f - o * ph (+ ph for up rows), f = row % 64, ph = 64 / s;
    owner r pairs slot lr (gate) with slot ph + lr (up) and writes output feature t * 64 + r * ph + lr.
    Stream-K form: the up row 64 + f is exchanged through entry f of the [64][16] area and read by the
    thread of gate row f. Either way every output feature f of a tile gets gate row f and up row 64 + f,
    once."""
    BM = 128
    for s in (2, 4, 8, 16):
        ph, per = (BM // 2) // s, BM // s
        slots = {}
        for row in range(BM):
            f = row % (BM // 2)
            o = f // ph
            slot = f - o * ph + (ph if row >= BM // 2 else 0)
            assert 0 <= slot < per and (o, slot) not in slots
            slots[(o, slot)] = row
        for r in range(s):
            for lr in range(ph):
                gate, up = slots[(r, lr)], slots[(r, ph + lr)]
                feature = r * ph + lr
                assert gate == feature and up == BM // 2 + feature
    for row in range(BM // 2, BM):  # stream-K exchange: the up thread's entry is its gate row's index
        assert row - BM // 2 == row % (BM // 2)
