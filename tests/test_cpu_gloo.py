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


def _check_functional_api(rank, world):
    import torch.distributed as dist

    import comm_opt_b200
    from comm_opt_b200.ops.reference import rel_err

    x, residual, gamma = _inputs(rank)
    res = residual.clone()
    out, new_res = comm_opt_b200.fused_allreduce_add_rmsnorm(x, res, gamma, 1e-6)
    assert new_res is res  # updated in place and returned
    xs = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(xs, x)
    h_ref = residual.double() + sum(t.double() for t in xs)
    out_ref = h_ref * torch.rsqrt(h_ref.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.double()
    assert rel_err(res, h_ref) < 1e-6 and rel_err(out, out_ref) < 1e-5
    g = torch.Generator().manual_seed(50 + rank)
    xb = torch.randn(4, 32, generator=g)
    w_row = 0.1 * torch.randn(4096, 32, generator=g)
    w_col = 0.1 * torch.randn(64, 4096, generator=g)
    res = residual.clone()
    z, _ = comm_opt_b200.layer_boundary(xb, w_row, res, gamma, w_col, 1e-6)
    y = xb.double() @ w_row.double().t()
    dist.all_reduce(y)
    h = residual.double() + y
    zr = (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * gamma.double()) @ w_col.double().t()
    assert rel_err(z, zr) < 1e-5 and rel_err(res, h) < 1e-6


def test_functional_api_gloo_world2():
    run_gloo(_check_functional_api, 2)


def test_functional_api_communicator_cache():
    """Capacity growth: a call beyond the cached communicator's capacity closes it and builds a larger one."""
    from comm_opt_b200 import api
    from comm_opt_b200.parallel.config import CommConfig

    made, closed = [], []

    class Fake:
        def __init__(self, group, cfg, device=None, dtype=None):
            self.max_rows, self.max_hidden = cfg.max_rows, cfg.max_hidden
            made.append((cfg.max_rows, cfg.max_hidden))

        def close(self):
            closed.append(1)

    api._COMMS.clear()
    x = torch.zeros(2, 8)
    cfg = CommConfig(max_rows=4, max_hidden=1024)
    c1 = api.communicator(x, 1024, 3, None, cfg, factory=Fake)
    assert api.communicator(x, 1024, 4, None, cfg, factory=Fake) is c1
    c2 = api.communicator(x, 2048, 9, None, cfg, factory=Fake)
    assert c2 is not c1 and closed == [1] and made == [(4, 1024), (9, 2048)]
    api._COMMS.clear()


def test_comm_config_env_and_dict():
    import pytest

    from comm_opt_b200.parallel.config import CommConfig

    c = CommConfig.from_env(env={"COB_MAX_ROWS": "64", "COB_PDL": "0", "COB_WAIT_TIMEOUT_MS": "250",
                                 "COB_HEAP_BACKEND": "ipc"})
    assert (c.max_rows, c.pdl, c.timeout_ms, c.backend) == (64, False, 250.0, "ipc")
    assert CommConfig.from_dict(c.kwargs()) == c
    with pytest.raises(ValueError):
        CommConfig.from_dict({"max_rowz": 3})
    with pytest.raises(ValueError):
        CommConfig(backend="nccl")
