// Bindings of the single-GPU decode kernels (see ops.h).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "check.h"

#include "common_host.h"
#include "gemm.h"
#include "ops.h"
#include "probes.h"
#include "types.h"

namespace {

int code_of(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kFloat: return cob::kF32;
    case torch::kHalf: return cob::kF16;
    case torch::kBFloat16: return cob::kBF16;
    default: COB_CHECK(false, "unsupported dtype ", std::string(c10::toString(t.scalar_type())));
  }
  return -1;
}

void ok(cudaError_t e, const char* what) { COB_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e)); }

void dense(const torch::Tensor& t, const char* n) {
  COB_CHECK(t.is_cuda() && t.is_contiguous(), n, " must be a contiguous CUDA tensor");
  COB_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, n, " must be 16-byte aligned");
}

cudaStream_t cur() { return at::cuda::getCurrentCUDAStream(); }

void py_rmsnorm(torch::Tensor x, torch::Tensor gamma, torch::Tensor out, double eps) {
  dense(x, "x");
  dense(gamma, "gamma");
  dense(out, "out");
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t H = x.size(-1);
  ok(cob::rmsnorm(x.data_ptr(), gamma.data_ptr(), out.data_ptr(), (int)(x.numel() / H), (int)H, (float)eps,
                  code_of(x), cur()),
     "rmsnorm");
}

void py_add_rmsnorm(torch::Tensor x, torch::Tensor residual, torch::Tensor gamma, torch::Tensor out, double eps) {
  dense(x, "x");
  dense(residual, "residual");
  dense(gamma, "gamma");
  dense(out, "out");
  const c10::cuda::CUDAGuard g(x.device());
  const int64_t H = x.size(-1);
  ok(cob::add_rmsnorm(x.data_ptr(), residual.data_ptr(), gamma.data_ptr(), out.data_ptr(), (int)(x.numel() / H),
                      (int)H, (float)eps, code_of(x), cur()),
     "add_rmsnorm");
}

void py_embedding(torch::Tensor ids, torch::Tensor table, torch::Tensor out) {
  dense(ids, "ids");
  dense(table, "table");
  dense(out, "out");
  COB_CHECK(ids.scalar_type() == torch::kInt32, "ids must be int32");
  const c10::cuda::CUDAGuard g(ids.device());
  ok(cob::embedding(ids.data_ptr<int32_t>(), table.data_ptr(), out.data_ptr(), (int)ids.numel(),
                    (int)table.size(1), code_of(table), cur()),
     "embedding");
}

void py_rope_append_kv(torch::Tensor qkv, torch::Tensor positions, torch::Tensor cos_t, torch::Tensor sin_t,
                       torch::Tensor block_tables, torch::Tensor q_out, torch::Tensor k_cache, torch::Tensor v_cache,
                       int64_t nq, int64_t nkv, c10::optional<torch::Tensor> bias) {
  for (auto* t : {&qkv, &positions, &cos_t, &sin_t, &block_tables, &q_out, &k_cache, &v_cache}) dense(*t, "arg");
  COB_CHECK(positions.scalar_type() == torch::kInt32 && block_tables.scalar_type() == torch::kInt32,
              "positions and block_tables must be int32");
  const int D = (int)k_cache.size(3), bs = (int)k_cache.size(2);
  const void* bptr = nullptr;
  if (bias.has_value()) {
    dense(*bias, "bias");
    COB_CHECK(bias->scalar_type() == qkv.scalar_type() && bias->numel() == (nq + 2 * nkv) * D,
              "bias must have the qkv dtype and (nq + 2 nkv) * head_dim elements");
    bptr = bias->data_ptr();
  }
  const c10::cuda::CUDAGuard g(qkv.device());
  ok(cob::rope_append_kv(qkv.data_ptr(), bptr, positions.data_ptr<int32_t>(), cos_t.data_ptr<float>(),
                         sin_t.data_ptr<float>(), block_tables.data_ptr<int32_t>(), (int)block_tables.size(1),
                         q_out.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), (int)qkv.size(0), (int)nq,
                         (int)nkv, D, bs, code_of(qkv), cur()),
     "rope_append_kv");
}

void py_silu_mul(torch::Tensor gu, torch::Tensor out, int64_t interleave) {
  dense(gu, "gu");
  dense(out, "out");
  COB_CHECK(gu.dim() == 2 && out.dim() == 2 && gu.size(0) == out.size(0) && gu.size(1) == 2 * out.size(1),
            "gu [M, 2I], out [M, I]");
  COB_CHECK(gu.scalar_type() == out.scalar_type(), "dtypes must match");
  const c10::cuda::CUDAGuard g(gu.device());
  ok(cob::silu_mul(gu.data_ptr(), out.data_ptr(), (int)gu.size(0), (int)out.size(1), code_of(gu), cur(),
                   (int)interleave),
     "silu_mul");
}

// keys: int64 [rows], zero before the first call (argmax_combine clears them)
void py_argmax_local(torch::Tensor logits, torch::Tensor keys, int64_t vocab_offset) {
  dense(logits, "logits");
  dense(keys, "keys");
  COB_CHECK(keys.scalar_type() == torch::kInt64 && keys.numel() == logits.size(0), "keys must be int64 [rows]");
  const c10::cuda::CUDAGuard g(logits.device());
  ok(cob::argmax_local(logits.data_ptr(), reinterpret_cast<unsigned long long*>(keys.data_ptr()), (int)logits.size(0),
                       (int)logits.size(1), (int)vocab_offset, code_of(logits), cur()),
     "argmax_local");
}

void py_argmax_combine(torch::Tensor gathered, torch::Tensor ids, int64_t world, c10::optional<torch::Tensor> positions,
                       c10::optional<torch::Tensor> seq_lens, c10::optional<torch::Tensor> local_keys) {
  dense(gathered, "gathered");
  dense(ids, "ids");
  COB_CHECK(gathered.scalar_type() == torch::kInt64 && gathered.numel() == world * ids.numel(),
              "gathered must be int64 [world, rows]");
  int32_t* pos = nullptr;
  int32_t* lens = nullptr;
  unsigned long long* lk = nullptr;
  if (positions.has_value()) {
    COB_CHECK(positions->scalar_type() == torch::kInt32 && positions->numel() == ids.numel(), "positions");
    pos = positions->data_ptr<int32_t>();
  }
  if (seq_lens.has_value()) {
    COB_CHECK(seq_lens->scalar_type() == torch::kInt32 && seq_lens->numel() == ids.numel(), "seq_lens");
    lens = seq_lens->data_ptr<int32_t>();
  }
  if (local_keys.has_value()) {
    COB_CHECK(local_keys->scalar_type() == torch::kInt64 && local_keys->numel() == ids.numel(), "local_keys");
    lk = reinterpret_cast<unsigned long long*>(local_keys->data_ptr());
  }
  const c10::cuda::CUDAGuard g(gathered.device());
  ok(cob::argmax_combine(reinterpret_cast<const unsigned long long*>(gathered.data_ptr()), ids.data_ptr<int32_t>(),
                         (int)ids.numel(), (int)world, pos, lens, lk, cur()),
     "argmax_combine");
}

int64_t py_attn_scratch_bytes(int64_t batch, int64_t nkv, int64_t splits, int64_t group, int64_t head_dim) {
  return (int64_t)cob::attn_scratch_bytes((int)batch, (int)nkv, (int)splits, (int)group, (int)head_dim);
}

// scratch: uint8 tensor of at least attn_scratch_bytes; its counter part must be zero before the
// first call (the kernel leaves it zero).
void py_decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_tables,
                         torch::Tensor seq_lens, torch::Tensor out, torch::Tensor scratch, int64_t splits,
                         int64_t pages_per_split, double scale, bool cluster, c10::optional<torch::Tensor> qkv,
                         c10::optional<torch::Tensor> qkv_bias, c10::optional<torch::Tensor> positions,
                         c10::optional<torch::Tensor> cos_t, c10::optional<torch::Tensor> sin_t) {
  for (auto* t : {&q, &k_cache, &v_cache, &block_tables, &seq_lens, &out, &scratch}) dense(*t, "arg");
  COB_CHECK(block_tables.scalar_type() == torch::kInt32 && seq_lens.scalar_type() == torch::kInt32,
              "block_tables and seq_lens must be int32");
  cob::AttnParams p = {};
  p.batch = (int)q.size(0);
  p.nq = (int)q.size(1);
  p.head_dim = (int)q.size(2);
  p.nkv = (int)k_cache.size(1);
  p.block_size = (int)k_cache.size(2);
  p.max_blocks_per_seq = (int)block_tables.size(1);
  p.splits = (int)splits;
  p.pages_per_split = (int)pages_per_split;
  p.scale = (float)scale;
  p.dtype = code_of(q);
  const int group = p.nq / p.nkv;
  const size_t need = cob::attn_scratch_bytes(p.batch, p.nkv, p.splits, group, p.head_dim);
  COB_CHECK((size_t)scratch.numel() * scratch.element_size() >= need, "attention scratch too small: need ", need);
  const size_t pairs = (size_t)p.batch * p.nkv;
  char* base = reinterpret_cast<char*>(scratch.data_ptr());
  p.part_o = reinterpret_cast<float*>(base);
  p.part_ml = reinterpret_cast<float*>(base + pairs * p.splits * group * p.head_dim * sizeof(float));
  p.counters = reinterpret_cast<int32_t*>(base + pairs * p.splits * group * p.head_dim * sizeof(float) +
                                          pairs * p.splits * group * 2 * sizeof(float));
  p.q = q.data_ptr();
  p.k_cache = k_cache.data_ptr();
  p.v_cache = v_cache.data_ptr();
  p.block_tables = block_tables.data_ptr<int32_t>();
  p.seq_lens = seq_lens.data_ptr<int32_t>();
  p.out = out.data_ptr();
  p.num_blocks = (int)k_cache.size(0);
  p.err = nullptr;
  p.cluster = cluster ? 1 : 0;
  if (qkv.has_value()) {  // RoPE + KV append of the new token inside the attention kernel
    COB_CHECK(positions.has_value() && cos_t.has_value() && sin_t.has_value(), "fused append needs positions, cos, sin");
    for (auto* t : {&*qkv, &*positions, &*cos_t, &*sin_t}) dense(*t, "fused append operand");
    COB_CHECK(qkv->scalar_type() == q.scalar_type() && qkv->dim() == 2 && qkv->size(0) == p.batch &&
                  qkv->size(1) == (int64_t)(p.nq + 2 * p.nkv) * p.head_dim,
              "qkv must be [batch, (nq + 2 nkv) * head_dim] of the query dtype");
    COB_CHECK(positions->scalar_type() == torch::kInt32 && positions->numel() >= p.batch, "positions: int32 [batch]");
    COB_CHECK(cos_t->scalar_type() == torch::kFloat && sin_t->scalar_type() == torch::kFloat &&
                  cos_t->size(-1) == p.head_dim / 2 && sin_t->size(-1) == p.head_dim / 2,
              "cos / sin: float32 [max_pos, head_dim / 2]");
    p.qkv = qkv->data_ptr();
    p.positions = positions->data_ptr<int32_t>();
    p.cos_t = cos_t->data_ptr<float>();
    p.sin_t = sin_t->data_ptr<float>();
    if (qkv_bias.has_value()) {
      dense(*qkv_bias, "qkv_bias");
      COB_CHECK(qkv_bias->scalar_type() == q.scalar_type() && qkv_bias->numel() == qkv->size(1), "qkv_bias size");
      p.qkv_bias = qkv_bias->data_ptr();
    }
  }
  const c10::cuda::CUDAGuard g(q.device());
  ok(cob::paged_decode_attention(p, cur()), "paged_decode_attention");
}

// y = x @ w^T on the tcgen05 tensor cores. `ws` float32 workspace, `ctr` int32 tile counters
// (zero-initialised, left zero). Returns {bn, tiles, ctas}.
std::vector<int64_t> py_gemm(torch::Tensor x, torch::Tensor w, torch::Tensor y, torch::Tensor ws, torch::Tensor ctr,
                             torch::Tensor err, int64_t ctas, bool pdl, bool small_smem, int64_t cluster_splits,
                             int64_t timeout_ns, int64_t packed_n, bool swiglu) {
  dense(x, "x");
  dense(w, "w");
  dense(err, "err");
  COB_CHECK(y.is_cuda() && y.stride(-1) == 1, "y must be row-major");
  // packed_n > 0: w is the packed layout [tiles, K / 64, 128, 64] of an [packed_n, K] weight
  const bool packed = packed_n > 0;
  const int64_t N = packed ? packed_n : w.size(0);
  if (packed)
    COB_CHECK(w.dim() == 4 && w.size(2) == 128 && w.size(3) == 64 && w.size(0) == (N + 127) / 128 &&
                  x.dim() == 2 && x.size(1) == w.size(1) * 64,
              "packed w must be [ceil(N / 128), K / 64, 128, 64] for x [M, K]");
  else
    COB_CHECK(x.dim() == 2 && w.dim() == 2 && x.size(1) == w.size(1), "x [M, K], w [N, K]");
  if (swiglu)
    COB_CHECK(y.size(0) == x.size(0) && 2 * y.size(1) == N, "y must be [M, N / 2] with the SwiGLU epilogue");
  else
    COB_CHECK(y.size(0) == x.size(0) && y.size(1) == N, "y must be [M, N]");
  COB_CHECK(x.scalar_type() == w.scalar_type() && y.scalar_type() == x.scalar_type(), "dtypes must match");
  COB_CHECK(err.scalar_type() == torch::kInt32 && ctr.scalar_type() == torch::kInt32, "err, ctr must be int32");
  COB_CHECK(ws.scalar_type() == torch::kFloat && ws.is_cuda() && ctr.is_cuda(), "ws must be float32 CUDA");
  const c10::cuda::CUDAGuard g(x.device());
  static int sms = 0;
  if (!sms) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, x.device().index());
  cob::GemmPlan p;
  ok(cob::gemm_decode(x.data_ptr(), w.data_ptr(), y.data_ptr(), (int)x.size(0), (int)N, (int)x.size(1),
                      (int)y.stride(0), code_of(x), ws.data_ptr<float>(), (size_t)ws.numel() * 4,
                      ctr.data_ptr<int32_t>(), (int)ctr.numel(), err.data_ptr<int32_t>(), sms, (int)ctas, pdl,
                      small_smem, (int)cluster_splits, (unsigned long long)timeout_ns, cur(), &p, packed, swiglu),
     "gemm_decode");
  return {p.bn, p.tiles, p.ctas};
}

std::vector<int64_t> py_gemm_plan(int64_t M, int64_t N, int64_t K, int64_t sms, int64_t ctas) {
  const cob::GemmPlan p = cob::plan_gemm((int)M, (int)N, (int)K, (int)sms, (int)ctas);
  return {p.bn, p.tiles, p.ctas, (int64_t)cob::gemm_workspace_bytes(p.ctas, p.bn)};
}

void py_rs_atomic_probe(std::vector<int64_t> bases, int64_t acc_off, int64_t ctr_off, torch::Tensor x, int64_t rank,
                        int64_t n, int64_t variant, int64_t emulate, int64_t x_rank_bytes, int64_t blocks,
                        int64_t timeout_ns, torch::Tensor err) {
  dense(x, "x");
  COB_CHECK(bases.size() >= 1 && bases.size() <= 8, "world must be 1..8");
  COB_CHECK(variant >= 0 && variant <= 3 && n > 0 && rank >= 0 && rank < (int64_t)bases.size(), "bad probe geometry");
  // input bytes the kernel reads: every rank's [world, n] slices (emulated ranks at x_rank_bytes apart),
  // or this rank's own slices on a real rank (no per-rank offset there)
  const int64_t es = variant <= 1 ? 4 : 2, W = (int64_t)bases.size();
  const int64_t need = emulate ? (W - 1) * x_rank_bytes + W * n * es : W * n * es;
  COB_CHECK(x.numel() * x.element_size() >= need && (emulate ? x_rank_bytes >= W * n * es : x_rank_bytes == 0),
            "x is smaller than the slices the probe reads (x_rank_bytes must be 0 on a real rank)");
  cob::RsProbeParams p = {};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<char*>(bases[i]);
  p.acc_off = acc_off;
  p.ctr_off = ctr_off;
  p.x = x.data_ptr();
  p.x_rank_bytes = x_rank_bytes;
  p.rank = (int)rank;
  p.world = (int)bases.size();
  p.n = (int)n;
  p.variant = (int)variant;
  p.emulate = (int)emulate;
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.err = err.data_ptr<int32_t>();
  const c10::cuda::CUDAGuard g(x.device());
  ok(cob::rs_atomic_probe(p, (int)blocks, cur()), "rs_atomic_probe");
}

std::vector<int64_t> py_clock_calibration(int64_t ns, int64_t device) {
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  auto out = torch::zeros({2}, torch::TensorOptions().dtype(torch::kInt64).device(torch::kCUDA, (c10::DeviceIndex)device));
  ok(cob::clock_calibration((unsigned long long)ns, reinterpret_cast<long long*>(out.data_ptr()), cur()), "clock_calibration");
  auto h = out.cpu();
  return {h[0].item<int64_t>(), h[1].item<int64_t>()};
}

std::vector<int64_t> py_prim_layout(int64_t world, int64_t n) {
  long long f = 0, st = 0, l = 0, nv = 0;
  const size_t total = cob::prim_heap_bytes((int)world, (int)n, &f, &st, &l, &nv);
  return {(int64_t)total, f, st, l, nv};
}

void py_prim_probe(std::vector<int64_t> bases, std::vector<int64_t> offs, int64_t rank, int64_t n, int64_t mode,
                   int64_t emulate, int64_t blocks, int64_t threads, int64_t timeout_ns, torch::Tensor bad,
                   torch::Tensor err, int64_t mc) {
  COB_CHECK(bases.size() >= 1 && bases.size() <= 8 && (offs.size() == 3 || offs.size() == 4),
            "world 1..8, offsets {flags, stage, land[, nvls]}");
  COB_CHECK(bad.is_cuda() && bad.scalar_type() == torch::kInt32 && err.is_cuda() && err.scalar_type() == torch::kInt32,
            "bad / err must be CUDA int32");
  cob::PrimParams p = {};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<char*>(bases[i]);
  p.flags_off = offs[0];
  p.stage_off = offs[1];
  p.land_off = offs[2];
  p.nvls_off = offs.size() == 4 ? offs[3] : 0;
  p.mc = reinterpret_cast<char*>(mc);
  p.rank = (int)rank;
  p.world = (int)bases.size();
  p.n = (int)n;
  p.mode = (int)mode;
  p.emulate = (int)emulate;
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.bad = reinterpret_cast<unsigned int*>(bad.data_ptr());
  p.err = err.data_ptr<int32_t>();
  COB_CHECK(bad.numel() >= (emulate ? p.world : 1), "bad must hold one word per local rank");
  const c10::cuda::CUDAGuard g(bad.device());
  ok(cob::prim_probe(p, (int)blocks, (int)threads, cur()), "prim_probe");
}

cob::LineProbeParams line_params(const std::vector<int64_t>& bases, int64_t heap_bytes, int64_t lines_off,
                                 int64_t n_lines, int64_t rank, int64_t target, int64_t mode, int64_t emulate,
                                 int64_t observer_blocks, int64_t writer_blocks, int64_t epoch, int64_t timeout_ns,
                                 const torch::Tensor& counters) {
  COB_CHECK(bases.size() >= 2 && bases.size() <= 8, "world must be 2..8");
  COB_CHECK(counters.is_cuda() && counters.scalar_type() == torch::kInt64 && counters.numel() >= 5,
            "counters must be a CUDA int64 tensor of 5 words");
  COB_CHECK(target >= 0 && target < (int64_t)bases.size(), "target rank out of range");
  COB_CHECK(lines_off >= 0 && lines_off % 128 == 0 && n_lines >= 1 && lines_off + n_lines * 128 <= heap_bytes,
            "lines [", lines_off, ", +", n_lines * 128, ") do not fit the ", heap_bytes, "-byte heap (or misaligned)");
  cob::LineProbeParams p = {};
  for (size_t i = 0; i < bases.size(); ++i) p.base[i] = reinterpret_cast<char*>(bases[i]);
  p.lines_off = lines_off;
  p.n_lines = n_lines;
  p.rank = (int)rank;
  p.world = (int)bases.size();
  p.target = (int)target;
  p.mode = (int)mode;
  p.emulate = (int)emulate;
  p.observer_blocks = (int)observer_blocks;
  p.writer_blocks = (int)writer_blocks;
  p.epoch = (unsigned int)epoch;
  p.timeout_ns = (unsigned long long)timeout_ns;
  p.counters = reinterpret_cast<unsigned long long*>(counters.data_ptr());
  return p;
}

void py_line_probe(std::vector<int64_t> bases, int64_t heap_bytes, int64_t lines_off, int64_t n_lines, int64_t rank,
                   int64_t target, int64_t mode, int64_t emulate, int64_t observer_blocks, int64_t writer_blocks,
                   int64_t epoch, int64_t timeout_ns, torch::Tensor counters, bool check) {
  const cob::LineProbeParams p = line_params(bases, heap_bytes, lines_off, n_lines, rank, target, mode, emulate,
                                             observer_blocks, writer_blocks, epoch, timeout_ns, counters);
  const c10::cuda::CUDAGuard g(counters.device());
  if (check)
    ok(cob::line_check(p, cur()), "line_check");
  else
    ok(cob::line_probe(p, cur()), "line_probe");
}

}  // namespace

void register_ops(pybind11::module& m) {
  m.def("line_probe", &py_line_probe);
  m.def("prim_layout", &py_prim_layout);
  m.def("prim_probe", &py_prim_probe, pybind11::arg("bases"), pybind11::arg("offs"), pybind11::arg("rank"),
        pybind11::arg("n"), pybind11::arg("mode"), pybind11::arg("emulate"), pybind11::arg("blocks"),
        pybind11::arg("threads"), pybind11::arg("timeout_ns"), pybind11::arg("bad"), pybind11::arg("err"),
        pybind11::arg("mc") = 0);
  m.def("rs_atomic_probe", &py_rs_atomic_probe);
  m.def("clock_calibration", &py_clock_calibration);
  m.def("gemm", &py_gemm);
  m.def("gemm_plan", &py_gemm_plan);
  m.def("rmsnorm", &py_rmsnorm);
  m.def("add_rmsnorm", &py_add_rmsnorm);
  m.def("embedding", &py_embedding);
  m.def("rope_append_kv", &py_rope_append_kv, pybind11::arg("qkv"), pybind11::arg("positions"), pybind11::arg("cos_t"),
        pybind11::arg("sin_t"), pybind11::arg("block_tables"), pybind11::arg("q_out"), pybind11::arg("k_cache"),
        pybind11::arg("v_cache"), pybind11::arg("nq"), pybind11::arg("nkv"), pybind11::arg("bias") = pybind11::none());
  m.def("silu_mul", &py_silu_mul, pybind11::arg("gu"), pybind11::arg("out"), pybind11::arg("interleave") = 0);
  m.def("argmax_local", &py_argmax_local);
  m.def("argmax_combine", &py_argmax_combine, pybind11::arg("gathered"), pybind11::arg("ids"),
        pybind11::arg("world"), pybind11::arg("positions") = pybind11::none(), pybind11::arg("seq_lens") = pybind11::none(),
        pybind11::arg("local_keys") = pybind11::none());
  m.def("set_pdl", [](bool on) { cob::pdl_flag() = on; });
  m.def("get_pdl", []() { return cob::pdl_flag(); });
  m.def(
      "set_gemm_stamps",
      [](int64_t ptr, int64_t stride) {
        cob::gemm_stamps() = reinterpret_cast<long long*>(ptr);
        cob::gemm_stamp_stride() = stride;
        cob::gemm_stamp_launches() = 0;
      },
      pybind11::arg("ptr"), pybind11::arg("stride") = 0);
  m.def("gemm_stamp_launches", []() { return (int64_t)cob::gemm_stamp_launches(); });
  m.def("set_l2_prefetch", [](int64_t tiles) { cob::l2_prefetch_tiles() = (int)std::max<int64_t>(0, tiles); });
  m.def("get_l2_prefetch", []() { return (int64_t)cob::l2_prefetch_tiles(); });
  m.def("set_attn_stages", [](int64_t n) {
    const int old = cob::attn_stage_mode();
    cob::attn_stage_mode() = (int)n;
    return (int64_t)old;
  });
  m.def("attn_scratch_bytes", &py_attn_scratch_bytes);
  m.def("attn_launch_smem_bytes", [](int64_t splits, int64_t group, int64_t head_dim, bool cluster, int64_t stages) {
    return (int64_t)cob::attn_launch_smem_bytes((int)splits, (int)group, (int)head_dim, cluster, (int)stages);
  });
  m.def("decode_attention", &py_decode_attention, pybind11::arg("q"), pybind11::arg("k_cache"),
        pybind11::arg("v_cache"), pybind11::arg("block_tables"), pybind11::arg("seq_lens"), pybind11::arg("out"),
        pybind11::arg("scratch"), pybind11::arg("splits"), pybind11::arg("pages_per_split"), pybind11::arg("scale"),
        pybind11::arg("cluster"), pybind11::arg("qkv") = pybind11::none(), pybind11::arg("qkv_bias") = pybind11::none(),
        pybind11::arg("positions") = pybind11::none(), pybind11::arg("cos") = pybind11::none(),
        pybind11::arg("sin") = pybind11::none());
}
