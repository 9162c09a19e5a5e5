"""CPU/gloo tier: world_size 2 correctness of fused all-reduce + residual add + RMSNorm.

Config (the reference's gloo correctness test): per-rank x [T=4, H=4096] fp32 ~N(0,1) (seed + rank), residual [4, 4096]
~N(0,1) (same on every rank), gamma = 1 + 0.1 N(0,1), eps = 1e-6. Output must equal
RMSNorm(sum_ranks(x) + residual) * gamma and the new residual must be returned.
"""
import torch

from conftest import run_gloo


def _inputs(rank, T=4, H=4096, dtype=torch.float32):
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(1234 + rank)).to(dtype)
    residual = torch.randn(T, H, generator=torch.Generator().manual_seed(99)).to(dtype)
    gamma = (1 + 0.1 * torch.randn(H, generator=torch.Generator().manual_seed(7))).to(dtype)
    return x, residual, gamma


def _check_oracle(rank, world):
    import torch.distributed as dist

    from comm_opt_b200.ops.reference import dist_fused_allreduce_add_rmsnorm_ref, rel_err
    from comm_opt_b200.parallel.cpu_collective import twoshot_fused_cpu

    x, residual, gamma = _inputs(rank)
    eps = 1e-6
    out, h = dist_fused_allreduce_add_rmsnorm_ref(x, residual, gamma, eps)
    # independent statement: gather every rank's x explicitly
    xs = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(xs, x)
    total = sum(t.double() for t in xs)
    h_ref = residual.double() + total
    out_ref = h_ref * torch.rsqrt(h_ref.pow(2).mean(-1, keepdim=True) + eps) * gamma.double()
    assert rel_err(h, h_ref) < 1e-6
    assert rel_err(out, out_ref) < 1e-6
    # the kernel's column-sharded two-shot decomposition gives the same answer
    out2, h2 = twoshot_fused_cpu(x, residual, gamma, eps)
    assert rel_err(h2, h_ref) < 1e-6
    assert rel_err(out2, out_ref) < 1e-5
    # bf16 inputs: within the reference's 2^-5 relative tolerance, outputs identical on all ranks
    xb, rb, gb = _inputs(rank, dtype=torch.bfloat16)
    out3, h3 = twoshot_fused_cpu(xb, rb, gb, eps)
    o_ref, h_ref3 = dist_fused_allreduce_add_rmsnorm_ref(xb, rb, gb, eps)
    assert rel_err(out3, o_ref) <= 2 ** -5 and rel_err(h3, h_ref3) <= 2 ** -5
    outs = [torch.empty_like(out3) for _ in range(world)]
    dist.all_gather(outs, out3)
    assert all(torch.equal(o, outs[0]) for o in outs)


def test_fused_oracle_gloo_world2():
    run_gloo(_check_oracle, 2)


def test_fused_oracle_gloo_world4():
    run_gloo(_check_oracle, 4)


def _check_layer_boundary(rank, world):
    import torch.distributed as dist

    from comm_opt_b200.ops.reference import rel_err
    from comm_opt_b200.parallel.cpu_collective import layer_boundary_cpu

    g = torch.Generator().manual_seed(100 + rank)
    M, K1, H, N, eps = 4, 64, 256, 96, 1e-5
    x = torch.randn(M, K1, generator=g).bfloat16()
    w_row = (0.1 * torch.randn(H, K1, generator=g)).bfloat16()
    w_col = (0.1 * torch.randn(N, H, generator=g)).bfloat16()
    shared = torch.Generator().manual_seed(5)
    residual = torch.randn(M, H, generator=shared).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=shared)).bfloat16()
    z, h = layer_boundary_cpu(x, w_row, residual, gamma, w_col, eps)
    # unfused statement: all-reduce of fp32 GEMM outputs, residual, RMSNorm, then the next GEMM
    y = x.double() @ w_row.double().t()
    dist.all_reduce(y)
    h_ref = residual.double() + y
    n_ref = h_ref * torch.rsqrt(h_ref.pow(2).mean(-1, keepdim=True) + eps) * gamma.double()
    z_ref = n_ref @ w_col.double().t()
    assert rel_err(h, h_ref) <= 2 ** -5 and rel_err(z, z_ref) <= 2 ** -5
    hs = [torch.empty_like(h) for _ in range(world)]
    dist.all_gather(hs, h)
    assert all(torch.equal(t, hs[0]) for t in hs)  # the new residual is identical on every rank


def test_layer_boundary_statement_gloo_world2():
    run_gloo(_check_layer_boundary, 2)
