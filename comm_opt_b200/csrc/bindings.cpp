// Python bindings of comm_opt_b200._C. Kernel sources are plain CUDA (no torch headers); this file
// only converts tensors to raw pointers, picks the current stream and turns error codes into
// exceptions.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "check.h"

#include <vector>

#include "fused_ar.h"
#include "fused_gemm.h"
#include "ops.h"
#include "tma_host.h"
#include "types.h"

namespace cob {
void fail(const std::string& m) { throw std::runtime_error(m); }
}  // namespace cob

namespace {

using cob::Layout;

std::vector<int64_t> layout_to_vec(const Layout& L) {
  return {L.state, L.flags, L.nvls,  L.land1,    L.rs,     L.ag,     L.agp,   L.stage,      L.hbuf,
          L.hpart, L.gather, L.total, L.world, L.max_rows, L.max_hv, L.sv_max, L.esize, L.max_gather};
}

Layout vec_to_layout(const std::vector<int64_t>& v) {
  COB_CHECK(v.size() == 18, "layout must have 18 fields");
  Layout L;
  L.state = v[0];
  L.flags = v[1];
  L.nvls = v[2];
  L.land1 = v[3];
  L.rs = v[4];
  L.ag = v[5];
  L.agp = v[6];
  L.stage = v[7];
  L.hbuf = v[8];
  L.hpart = v[9];
  L.gather = v[10];
  L.total = v[11];
  L.world = (int)v[12];
  L.max_rows = (int)v[13];
  L.max_hv = (int)v[14];
  L.sv_max = (int)v[15];
  L.esize = (int)v[16];
  L.max_gather = (int)v[17];
  return L;
}

int dtype_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kFloat: return cob::kF32;
    case torch::kHalf: return cob::kF16;
    case torch::kBFloat16: return cob::kBF16;
    default: COB_CHECK(false, "unsupported dtype ", std::string(c10::toString(t.scalar_type())));
  }
  return -1;
}

void check_cuda(cudaError_t e, const char* what) {
  COB_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

void check_dense(const torch::Tensor& t, const char* name) {
  COB_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  COB_CHECK(t.is_contiguous(), name, " must be contiguous");
  COB_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

std::vector<int64_t> py_plan_layout(int64_t world, int64_t max_rows, int64_t max_hidden, int64_t esize,
                                    int64_t max_gather) {
  return layout_to_vec(cob::plan_layout((int)world, (int)max_rows, (int)max_hidden, (int)esize, (int)max_gather));
}

void py_init_heap(torch::Tensor heap, std::vector<int64_t> layout, int64_t dtype) {
  check_dense(heap, "heap");
  const Layout L = vec_to_layout(layout);
  COB_CHECK(heap.numel() * heap.element_size() >= L.total, "heap smaller than layout");
  const c10::cuda::CUDAGuard g(heap.device());
  check_cuda(cob::init_heap(reinterpret_cast<char*>(heap.data_ptr()), L, (int)dtype,
                            at::cuda::getCurrentCUDAStream()),
             "init_heap");
}

// Returns {status, variant, blocks, threads, cluster}; status is a cudaError_t of the configuration
// check (the Python side raises with the resolved geometry in the message).
std::vector<int64_t> py_fused_ar(std::vector<int64_t> bases, int64_t mc, std::vector<int64_t> layout,
                                 torch::Tensor x, torch::Tensor residual, torch::Tensor gamma, torch::Tensor out,
                                 int64_t rank, int64_t rows, int64_t hidden, double eps, int64_t variant,
                                 int64_t blocks, int64_t threads, int64_t cluster, int64_t emulate, int64_t pdl,
                                 int64_t norm, int64_t timeout_ns, int64_t x_rs, int64_t res_rs, int64_t out_rs,
                                 bool dry_run, c10::optional<torch::Tensor> stamps) {
  cob::ARParams p = {};
  COB_CHECK(bases.size() >= 2 && bases.size() <= cob::kMaxWorld, "world must be 2..8");
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<char*>(bases[i]);
  p.mc = reinterpret_cast<char*>(mc);
  p.L = vec_to_layout(layout);
  check_dense(x, "x");
  check_dense(out, "out");
  COB_CHECK(out.scalar_type() == x.scalar_type(), "out dtype must match x");
  if (norm) {
    check_dense(residual, "residual");
    check_dense(gamma, "gamma");
    COB_CHECK(residual.scalar_type() == x.scalar_type() && gamma.scalar_type() == x.scalar_type(),
                "x, residual and gamma must share a dtype");
    p.residual = residual.data_ptr();
    p.gamma = gamma.data_ptr();
  }
  p.x = x.data_ptr();
  p.out = out.data_ptr();
  p.x_rs = x_rs;
  p.res_rs = res_rs;
  p.out_rs = out_rs;
  p.rank = (int)rank;
  p.world = (int)bases.size();
  p.rows = (int)rows;
  p.hidden = (int)hidden;
  p.eps = (float)eps;
  p.variant = (int)variant;
  p.blocks = (int)blocks;
  p.threads = (int)threads;
  p.cluster = (int)cluster;
  p.emulate = (int)emulate;
  p.pdl = (int)pdl;
  p.norm = (int)norm;
  p.dtype = dtype_code(x);
  p.timeout_ns = (unsigned long long)timeout_ns;
  if (stamps.has_value()) {
    COB_CHECK(stamps->is_cuda() && stamps->scalar_type() == torch::kInt64 && stamps->dim() == 4 &&
                  stamps->size(2) == cob::kMaxBlocks && stamps->size(3) == cob::kStampPhases,
              "stamps must be int64 [ranks, cap, kMaxBlocks, kStampPhases]");
    p.stamps = reinterpret_cast<long long*>(stamps->data_ptr());
    p.stamp_cap = (int)stamps->size(1);
  }
  COB_CHECK(p.L.world == p.world, "layout world ", p.L.world, " != ", p.world);
  COB_CHECK(p.L.esize == (int)x.element_size(), "communicator dtype size ", p.L.esize, " != input ",
              x.element_size());
  COB_CHECK(p.variant >= 1 && p.variant < cob::kNumVariants, "variant must be resolved by the caller");
  const c10::cuda::CUDAGuard g(x.device());
  int sms = 0;
  check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.device().index()), "sm count");
  const cudaError_t rc = cob::resolve_config(p, sms);
  if (rc == cudaSuccess && !dry_run)
    check_cuda(cob::launch_fused_ar(p, at::cuda::getCurrentCUDAStream()), "fused_ar launch");
  return {(int64_t)rc, p.variant, p.blocks, p.threads, p.cluster};
}

void py_allgather_u32(std::vector<int64_t> bases, std::vector<int64_t> layout, torch::Tensor in, torch::Tensor out,
                      int64_t rank, int64_t n, int64_t emulate, int64_t timeout_ns, int64_t in_rs, int64_t out_rs) {
  cob::GatherParams p = {};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<char*>(bases[i]);
  p.L = vec_to_layout(layout);
  check_dense(in, "in");
  check_dense(out, "out");
  COB_CHECK(in.element_size() == 4 && out.element_size() == 4, "32-bit words only");
  p.in = reinterpret_cast<const uint32_t*>(in.data_ptr());
  p.out = reinterpret_cast<uint32_t*>(out.data_ptr());
  p.in_rs = in_rs;
  p.out_rs = out_rs;
  p.rank = (int)rank;
  p.world = (int)bases.size();
  p.n = (int)n;
  p.emulate = (int)emulate;
  p.timeout_ns = (unsigned long long)timeout_ns;
  const c10::cuda::CUDAGuard g(in.device());
  check_cuda(cob::launch_allgather_u32(p, at::cuda::getCurrentCUDAStream()), "allgather_u32");
}


// Layer-boundary fused GEMMs. kind 0 = gemm_push (x -> landing buffers of every rank),
// kind 1 = ar_norm_gemm (landing buffers + residual + gamma -> y). Weights w are [ranks * N, K]
// (emulate: every rank's weights stacked), x [ranks * M, K]. Returns {bn, tiles, splits, kps, xctas}.
std::vector<int64_t> py_fused_gemm(int64_t kind, std::vector<int64_t> bases, std::vector<int64_t> layout,
                                   torch::Tensor w, c10::optional<torch::Tensor> x,
                                   c10::optional<torch::Tensor> residual, c10::optional<torch::Tensor> gamma,
                                   c10::optional<torch::Tensor> y, c10::optional<torch::Tensor> act,
                                   c10::optional<torch::Tensor> flags, c10::optional<torch::Tensor> pss,
                                   torch::Tensor err, int64_t rank, int64_t M, int64_t N, int64_t K, double eps,
                                   int64_t emulate, int64_t splits, int64_t pdl, int64_t timeout_ns,
                                   int64_t res_rs, bool dry_run, int64_t epi,
                                   c10::optional<torch::Tensor> positions, c10::optional<torch::Tensor> cos_t,
                                   c10::optional<torch::Tensor> sin_t, c10::optional<torch::Tensor> block_tables,
                                   c10::optional<torch::Tensor> k_cache, c10::optional<torch::Tensor> v_cache,
                                   int64_t nq, int64_t nkv, bool packed) {
  cob::FusedGemmParams p = {};
  COB_CHECK(bases.size() >= 1 && bases.size() <= cob::kMaxWorld, "world must be 1..8");
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<char*>(bases[i]);
  p.L = vec_to_layout(layout);
  p.world = (int)bases.size();
  p.rank = (int)rank;
  p.emulate = (int)emulate;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.eps = (float)eps;
  p.timeout_ns = (unsigned long long)timeout_ns;
  const int ranks = emulate ? p.world : 1;
  check_dense(w, "w");
  check_dense(err, "err");
  COB_CHECK(w.scalar_type() == torch::kBFloat16, "fused GEMMs take bf16 weights");
  const int64_t wtiles = (N + 127) / 128;
  if (packed)  // [ranks * ceil(N / 128), K / 64, 128, 64] blocks (see gemm.h)
    COB_CHECK(K % 64 == 0 && w.numel() == (int64_t)ranks * wtiles * 128 * K,
              "packed w must hold ranks * ceil(N / 128) * 128 * K elements");
  else
    COB_CHECK(w.numel() == (int64_t)ranks * N * K, "w must hold ranks * N * K elements");
  p.wp = packed ? reinterpret_cast<const uint8_t*>(w.data_ptr()) : nullptr;
  p.w_tiles = (int)wtiles;
  COB_CHECK(err.scalar_type() == torch::kInt32, "err must be int32");
  COB_CHECK(p.L.world == p.world && p.L.esize == 2, "communicator layout must be bf16 with this world");
  p.err = reinterpret_cast<int*>(err.data_ptr());
  const c10::cuda::CUDAGuard g(w.device());
  int sms = 0;
  check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, w.device().index()), "sm count");
  COB_CHECK(epi >= 0 && epi <= 2 && (kind == 1 || epi == 0), "epilogue 0 plain, 1 swiglu, 2 rope_kv (consumer only)");
  p.epi = (int)epi;
  cob::FusedGemmPlan pl =
      cob::plan_fused_gemm((int)M, (int)N, (int)K, (int)splits, std::max(1, sms / ranks), kind == 1, (int)epi);
  if (kind == 1 && splits <= 0 && !dry_run) {
    // automatic plan of the consumer: fewer K-splits while the occupancy bound says its clusters do not
    // all fit at once (launch_ar_norm_gemm would reject the grid)
    while (pl.splits > 1) {
      const int cap = cob::ar_norm_gemm_resident_clusters(pl.bn, pl.splits);
      if (cap < 0 || (long long)pl.xctas * ranks <= cap) break;
      const int fewer = pl.splits / 2;
      if (epi != cob::kEpiPlain && fewer < 2) break;
      pl = cob::plan_fused_gemm((int)M, (int)N, (int)K, fewer, std::max(1, sms / ranks), true, (int)epi);
    }
  }
  if (dry_run) return {pl.bn, pl.tiles, pl.splits, pl.kps, pl.xctas};
  COB_CHECK(pl.splits > 0, "no launch geometry supports this epilogue for [", M, ", ", N, ", ", K, "]");
  if (epi == cob::kEpiRopeKv) {
    COB_CHECK(positions.has_value() && cos_t.has_value() && sin_t.has_value() && block_tables.has_value() &&
                  k_cache.has_value() && v_cache.has_value(),
              "rope_kv epilogue needs positions, cos, sin, block_tables, k_cache, v_cache");
    COB_CHECK(positions->scalar_type() == torch::kInt32 && block_tables->scalar_type() == torch::kInt32 &&
                  cos_t->scalar_type() == torch::kFloat && sin_t->scalar_type() == torch::kFloat &&
                  cos_t->size(-1) == 64 && k_cache->scalar_type() == torch::kBFloat16 &&
                  v_cache->scalar_type() == torch::kBFloat16 && k_cache->size(-1) == 128,
              "rope_kv operand types / shapes (head_dim 128, bf16 caches [blocks, nkv, bs, 128])");
    for (auto* t : {&*positions, &*cos_t, &*sin_t, &*block_tables, &*k_cache, &*v_cache}) check_dense(*t, "rope_kv operand");
    p.positions = positions->data_ptr<int32_t>();
    p.cos_t = cos_t->data_ptr<float>();
    p.sin_t = sin_t->data_ptr<float>();
    p.block_tables = block_tables->data_ptr<int32_t>();
    p.max_blocks = (int)block_tables->size(-1);
    p.k_cache = k_cache->data_ptr();
    p.v_cache = v_cache->data_ptr();
    p.nq = (int)nq;
    p.nkv = (int)nkv;
    p.bs = (int)k_cache->size(-2);
    p.cache_rs = emulate ? k_cache->numel() / ranks : 0;
  }
  CUtensorMap tw = {}, tb;
  if (!packed)
    check_cuda(cob::tensor_map_2d(w.data_ptr(), (uint64_t)ranks * N, (uint64_t)K, (uint64_t)K * 2, 128, 64, true, &tw),
               "weight tensor map");
  cudaError_t rc;
  if (kind == 0) {
    COB_CHECK(x.has_value(), "gemm_push needs x");
    check_dense(*x, "x");
    COB_CHECK(x->scalar_type() == torch::kBFloat16 && x->numel() == (int64_t)ranks * M * K, "x must be bf16 [ranks*M, K]");
    check_cuda(cob::tensor_map_2d(x->data_ptr(), (uint64_t)ranks * M, (uint64_t)K, (uint64_t)K * 2, (uint32_t)pl.bn, 64,
                                  true, &tb),
               "x tensor map");
    rc = cob::launch_gemm_push(p, tw, tb, pl, ranks, pdl != 0, at::cuda::getCurrentCUDAStream());
  } else {
    COB_CHECK(residual.has_value() && gamma.has_value() && y.has_value() && act.has_value() && flags.has_value() &&
                  pss.has_value(),
              "ar_norm_gemm needs residual, gamma, y, act, flags, pss");
    for (auto* t : {&*residual, &*gamma, &*y, &*act, &*flags, &*pss}) check_dense(*t, "fused GEMM operand");
    COB_CHECK(residual->scalar_type() == torch::kBFloat16 && gamma->scalar_type() == torch::kBFloat16 &&
                  y->scalar_type() == torch::kBFloat16 && act->scalar_type() == torch::kBFloat16,
              "residual, gamma, y, act must be bf16");
    const int64_t ycols = epi == cob::kEpiSwiglu ? N / 2 : (epi == cob::kEpiRopeKv ? nq * 128 : N);
    COB_CHECK(residual->numel() >= (int64_t)ranks * M * K && gamma->numel() == K &&
                  y->numel() >= (int64_t)ranks * M * ycols,
              "residual / gamma / y sizes");
    COB_CHECK(act->dim() == 2 && act->size(1) == K && act->size(0) % ranks == 0, "act must be [ranks * rows, K]");
    COB_CHECK(flags->scalar_type() == torch::kInt32 && flags->numel() >= (int64_t)ranks * cob::kMaxPieces,
              "flags must be int32 [ranks, kMaxPieces]");
    p.act_rows = (int)(act->size(0) / ranks);
    COB_CHECK(pss->scalar_type() == torch::kFloat && pss->numel() >= (int64_t)ranks * cob::kMaxPieces * p.act_rows,
              "pss must be float32 [ranks, kMaxPieces, rows]");
    p.residual = residual->data_ptr();
    p.gamma = gamma->data_ptr();
    p.Y = y->data_ptr();
    p.act = act->data_ptr();
    p.flags = reinterpret_cast<uint32_t*>(flags->data_ptr());
    p.pss = reinterpret_cast<float*>(pss->data_ptr());
    p.res_rs = res_rs;
    check_cuda(cob::tensor_map_2d(act->data_ptr(), (uint64_t)act->size(0), (uint64_t)K, (uint64_t)K * 2,
                                  (uint32_t)pl.bn, 64, true, &tb),
               "act tensor map");
    rc = cob::launch_ar_norm_gemm(p, tw, tb, pl, ranks, pdl != 0, at::cuda::getCurrentCUDAStream());
  }
  check_cuda(rc, kind == 0 ? "gemm_push launch" : "ar_norm_gemm launch");
  return {pl.bn, pl.tiles, pl.splits, pl.kps, pl.xctas};
}

}  // namespace

namespace {
// Host geometry of one fused all-reduce call (no device work): {status, variant, blocks, threads, cluster}.
std::vector<int64_t> py_fused_ar_config(std::vector<int64_t> layout, int64_t world, int64_t rows, int64_t hidden,
                                        int64_t dtype, int64_t variant, int64_t blocks, int64_t threads,
                                        int64_t cluster, int64_t emulate, int64_t sms, bool have_mc) {
  cob::ARParams p = {};
  p.L = vec_to_layout(layout);
  p.world = (int)world;
  p.rows = (int)rows;
  p.hidden = (int)hidden;
  p.dtype = (int)dtype;
  p.variant = (int)variant;
  p.blocks = (int)blocks;
  p.threads = (int)threads;
  p.cluster = (int)cluster;
  p.emulate = (int)emulate;
  p.mc = have_mc ? reinterpret_cast<char*>(1) : nullptr;  // only tested for null
  const cudaError_t rc = cob::resolve_config(p, (int)sms);
  return {(int64_t)rc, p.variant, p.blocks, p.threads, p.cluster};
}

// Host planner of the layer-boundary GEMMs (no device work): {bn, tiles, splits, kps, xctas, ctas, smem}.
std::vector<int64_t> py_fused_gemm_plan(int64_t M, int64_t N, int64_t K, int64_t splits, int64_t sms,
                                        bool consumer, int64_t epi) {
  const cob::FusedGemmPlan p = cob::plan_fused_gemm((int)M, (int)N, (int)K, (int)splits, (int)sms, consumer, (int)epi);
  return {p.bn, p.tiles, p.splits, p.kps, p.xctas, p.ctas, p.smem};
}
}  // namespace

void register_ops(pybind11::module& m);  // ops_bindings.cpp
void register_ipc(pybind11::module& m);  // ipc_bindings.cpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "comm_opt_b200 native kernels (sm_100a)";
  m.def("plan_layout", &py_plan_layout);
  m.def("init_heap", &py_init_heap);
  m.def("fused_ar", &py_fused_ar, pybind11::arg("bases"), pybind11::arg("mc"), pybind11::arg("layout"),
        pybind11::arg("x"), pybind11::arg("residual"), pybind11::arg("gamma"), pybind11::arg("out"),
        pybind11::arg("rank"), pybind11::arg("rows"), pybind11::arg("hidden"), pybind11::arg("eps"),
        pybind11::arg("variant"), pybind11::arg("blocks"), pybind11::arg("threads"), pybind11::arg("cluster"),
        pybind11::arg("emulate"), pybind11::arg("pdl"), pybind11::arg("norm"), pybind11::arg("timeout_ns"),
        pybind11::arg("x_rs"), pybind11::arg("res_rs"), pybind11::arg("out_rs"), pybind11::arg("dry_run"),
        pybind11::arg("stamps") = pybind11::none());
  m.attr("kStampPhases") = cob::kStampPhases;
  m.def("allgather_u32", &py_allgather_u32);
  m.attr("kMaxBlocks") = cob::kMaxBlocks;
  m.attr("kMaxWorld") = cob::kMaxWorld;
  m.attr("kRankStateBytes") = (int64_t)sizeof(cob::RankState);
  m.def("fused_gemm", &py_fused_gemm, pybind11::arg("kind"), pybind11::arg("bases"), pybind11::arg("layout"),
        pybind11::arg("w"), pybind11::arg("x") = pybind11::none(), pybind11::arg("residual") = pybind11::none(),
        pybind11::arg("gamma") = pybind11::none(), pybind11::arg("y") = pybind11::none(),
        pybind11::arg("act") = pybind11::none(), pybind11::arg("flags") = pybind11::none(),
        pybind11::arg("pss") = pybind11::none(), pybind11::arg("err"), pybind11::arg("rank"), pybind11::arg("M"),
        pybind11::arg("N"), pybind11::arg("K"), pybind11::arg("eps"), pybind11::arg("emulate"),
        pybind11::arg("splits"), pybind11::arg("pdl"), pybind11::arg("timeout_ns"), pybind11::arg("res_rs"),
        pybind11::arg("dry_run"), pybind11::arg("epi") = 0, pybind11::arg("positions") = pybind11::none(),
        pybind11::arg("cos") = pybind11::none(), pybind11::arg("sin") = pybind11::none(),
        pybind11::arg("block_tables") = pybind11::none(), pybind11::arg("k_cache") = pybind11::none(),
        pybind11::arg("v_cache") = pybind11::none(), pybind11::arg("nq") = 0, pybind11::arg("nkv") = 0,
        pybind11::arg("packed") = false);
  m.attr("kMaxPieces") = cob::kMaxPieces;
  m.def("fused_gemm_plan", &py_fused_gemm_plan);
  m.def("ar_norm_gemm_resident_clusters",
        [](int64_t bn, int64_t splits) { return (int64_t)cob::ar_norm_gemm_resident_clusters((int)bn, (int)splits); });
  m.def("fused_ar_config", &py_fused_ar_config);
  register_ops(m);
  register_ipc(m);
}
