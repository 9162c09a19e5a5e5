// Decode-shaped GEMM on the 5th-generation tensor cores: Y[M, N] = X[M, K] * W[N, K]^T, M small.
//
// Swap-AB: a CTA owns 128 output features (the tcgen05 M dimension) and all M <= 256 batch rows
// (the tcgen05 N dimension, padded to 16..256), so the weight matrix - the bytes that bound decode -
// streams through shared memory exactly once:
//   warp 0 / one thread : TMA producer. Weight tiles (128 x 64, 128-byte swizzle) for the first ring
//                         slots are issued BEFORE the programmatic-dependent-launch wait (weights do
//                         not depend on the previous kernel); activation tiles after it.
//   warp 1 / one thread : tcgen05.mma issuer, fp32 accumulator in TMEM (BN columns), releases ring
//                         slots with tcgen05.commit -> mbarrier.
//   all 4 warps         : epilogue, tcgen05.ld of their 32 TMEM lanes, bf16 stores.
// Split-K: when there are fewer output tiles than SMs, the K range is split over a thread-block
// cluster (<= 8 CTAs along grid.y); partial tiles are summed through distributed shared memory in a
// fixed order (deterministic, no global workspace).
// Every mbarrier wait is bounded by %globaltimer; a timeout sets *err and the CTA drains and exits.
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <unordered_map>

#include "gemm.h"
#include "sm100.cuh"

namespace cob {
namespace {

namespace cg = cooperative_groups;
using namespace sm100;

constexpr int BM = 128, BK = 64, kThreads = 128;

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;  // 16 KB weight tile
  static constexpr int B_BYTES = BN * BK * 2;  // activation tile
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN <= 32 ? 8 : (BN <= 64 ? 6 : (BN <= 128 ? 5 : 4));
  static constexpr int PIPE = STAGES * STAGE;
  static constexpr int RED_STRIDE = BN + 1;  // fp32 partial row stride (bank-conflict padding)
  static constexpr int RED_BYTES = BM * RED_STRIDE * 4;
  static constexpr int BODY = PIPE > RED_BYTES ? PIPE : RED_BYTES;
  static constexpr int SMEM = BODY + 1024 + 256;  // alignment slack + barriers
  static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
};

template <bool BF16>
__device__ __forceinline__ void store_out(void* Y, size_t idx, float v) {
  if (BF16)
    reinterpret_cast<__nv_bfloat16*>(Y)[idx] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<__half*>(Y)[idx] = __float2half_rn(v);
}

template <int BN, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_swapab(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, void* Y, int M,
                  int N, int K, int kps, int ldy, int* err, unsigned long long timeout_ns) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::BODY);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* s_fail = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* s_issued = const_cast<int*>(s_fail) + 1;
  int* s_consumed = s_issued + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BM;
  const int KT = (K + BK - 1) / BK;
  const int kt0 = blockIdx.y * kps;
  const int nk = min(KT, kt0 + kps) - kt0;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmW);
    prefetch_tmap(&tmX);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *s_fail = 0;
    *s_issued = 0;
    *s_consumed = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    const int pre = min(C::STAGES, nk);
    for (int i = 0; i < pre; ++i) {
      mbar_arrive_expect_tx(&full[i], C::STAGE);
      tma_load_2d(sA + i * C::A_BYTES, &tmW, &full[i], (kt0 + i) * BK, n0);
    }
    pdl_wait();  // activations come from the previous kernel
    for (int i = 0; i < pre; ++i) tma_load_2d(sB + i * C::B_BYTES, &tmX, &full[i], (kt0 + i) * BK, 0);
    int issued = pre;
    for (int i = pre; i < nk; ++i) {
      const int s = i % C::STAGES;
      if (!mbar_wait(&empty[s], ((i / C::STAGES) & 1) ^ 1, timeout_ns) || *s_fail) {
        *s_fail = 1;
        break;
      }
      mbar_arrive_expect_tx(&full[s], C::STAGE);
      tma_load_2d(sA + s * C::A_BYTES, &tmW, &full[s], (kt0 + i) * BK, n0);
      tma_load_2d(sB + s * C::B_BYTES, &tmX, &full[s], (kt0 + i) * BK, 0);
      issued = i + 1;
    }
    *s_issued = issued;
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_f16(BM, BN, BF16);
    int consumed = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % C::STAGES;
      if (!mbar_wait(&full[s], (i / C::STAGES) & 1, timeout_ns) || *s_fail) {
        *s_fail = 1;
        break;
      }
      tc_fence_after();
      const uint32_t a = smem_addr(sA + s * C::A_BYTES), b = smem_addr(sB + s * C::B_BYTES);
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk)
        mma_f16(tmem, desc_k_sw128(a + kk * 32), desc_k_sw128(b + kk * 32), idesc, (i | kk) != 0);
      mma_commit(&empty[s]);
      consumed = i + 1;
    }
    *s_consumed = consumed;
    mma_commit(accum);
  }

  // ---------------------------------------------------------------- epilogue (all 4 warps)
  if (!mbar_wait(accum, 0, timeout_ns)) *s_fail = 1;
  __syncwarp();  // tcgen05.ld below is .sync.aligned: the warp must be converged
  tc_fence_after();
  pdl_trigger();
  const int row = warp * 32 + lane;
  const int n = n0 + row;
  const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16);
  const int mcols = min(M, BN);
  if (gridDim.y == 1) {
    for (int c0 = 0; c0 < mcols; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (n < N) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (c0 + j < M) store_out<BF16>(Y, (size_t)(c0 + j) * ldy + n, v[j]);
      }
    }
  } else {
    // split-K: partial tile -> own shared memory -> sum over the cluster through DSMEM
    cg::cluster_group cluster = cg::this_cluster();
    float* red = reinterpret_cast<float*>(smem);
    __syncthreads();  // every MMA read of the ring has completed (accum), reuse it
    for (int c0 = 0; c0 < mcols; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) red[row * C::RED_STRIDE + c0 + j] = v[j];
    }
    cluster.sync();
    const int cs = gridDim.y, r = blockIdx.y;
    const int per = (BM + cs - 1) / cs, r0 = r * per, r1 = min(BM, r0 + per), nr = r1 - r0;
    for (int idx = threadIdx.x; idx < nr * mcols; idx += kThreads) {
      const int rr = r0 + idx % nr, b = idx / nr;
      float acc = 0.f;
      for (int c = 0; c < cs; ++c) acc += cluster.map_shared_rank(red, c)[rr * C::RED_STRIDE + b];
      if (n0 + rr < N) store_out<BF16>(Y, (size_t)b * ldy + n0 + rr, acc);
    }
    cluster.sync();
  }

  // ---------------------------------------------------------------- teardown
  __syncthreads();
  if (threadIdx.x == 0 && *s_fail) {
    atomicOr(err, 1);
    // drain TMA loads that were issued but never consumed before the shared memory goes away
    for (int i = *s_consumed; i < *s_issued; ++i) mbar_wait(&full[i % C::STAGES], (i / C::STAGES) & 1, timeout_ns);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------------------ tensor maps (host)
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct MapKey {
  uint64_t ptr;
  int rows, cols, box_rows, bf16;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && box_rows == o.box_rows && bf16 == o.bf16;
  }
};
struct MapHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uint64_t>()(k.ptr) ^ ((size_t)k.rows * 1000003u) ^ ((size_t)k.cols << 20) ^
           ((size_t)k.box_rows << 40) ^ (size_t)k.bf16;
  }
};

// Row-major [rows, cols] 16-bit matrix, box = 64 columns (128 bytes, one swizzle span) x box_rows.
cudaError_t tensor_map(const void* ptr, int rows, int cols, int box_rows, bool bf16, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapHash> cache;
  const MapKey key{reinterpret_cast<uint64_t>(ptr), rows, cols, box_rows, bf16 ? 1 : 0};
  std::lock_guard<std::mutex> g(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  auto enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (cols * 2) % 16) return cudaErrorMisalignedAddress;
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(&m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                         const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (cache.size() > 8192) cache.clear();
  cache.emplace(key, m);
  *out = m;
  return cudaSuccess;
}

template <int BN, bool BF16>
cudaError_t launch_bn(const CUtensorMap& mw, const CUtensorMap& mx, void* Y, int M, int N, int K, int kps, int splits,
                      int ldy, int* err, unsigned long long timeout_ns, bool pdl, cudaStream_t stream) {
  using C = Cfg<BN>;
  auto fn = k_gemm_swapab<BN, BF16>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((N + BM - 1) / BM, splits, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (splits > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 1;
    attrs[na].val.clusterDim.y = splits;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, fn, mw, mx, Y, M, N, K, kps, ldy, err, timeout_ns);
}

template <bool BF16>
cudaError_t launch_typed(const CUtensorMap& mw, const CUtensorMap& mx, int bn, void* Y, int M, int N, int K, int kps,
                         int splits, int ldy, int* err, unsigned long long t, bool pdl, cudaStream_t s) {
  switch (bn) {
    case 16: return launch_bn<16, BF16>(mw, mx, Y, M, N, K, kps, splits, ldy, err, t, pdl, s);
    case 32: return launch_bn<32, BF16>(mw, mx, Y, M, N, K, kps, splits, ldy, err, t, pdl, s);
    case 64: return launch_bn<64, BF16>(mw, mx, Y, M, N, K, kps, splits, ldy, err, t, pdl, s);
    case 128: return launch_bn<128, BF16>(mw, mx, Y, M, N, K, kps, splits, ldy, err, t, pdl, s);
    case 256: return launch_bn<256, BF16>(mw, mx, Y, M, N, K, kps, splits, ldy, err, t, pdl, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

GemmPlan plan_gemm(int M, int N, int K, int num_sms, int splits_override) {
  GemmPlan p = {};
  p.bn = M <= 16 ? 16 : (M <= 32 ? 32 : (M <= 64 ? 64 : (M <= 128 ? 128 : 256)));
  const int tiles = (N + BM - 1) / BM, KT = (K + BK - 1) / BK;
  int s = splits_override > 0 ? splits_override : (tiles >= num_sms ? 1 : std::max(1, num_sms / tiles));
  s = std::max(1, std::min(std::min(s, 8), KT));
  p.kps = (KT + s - 1) / s;
  p.splits = (KT + p.kps - 1) / p.kps;
  p.tiles = tiles;
  return p;
}

cudaError_t gemm_decode(const void* X, const void* W, void* Y, int M, int N, int K, int ldy, int dtype, int* err,
                        int num_sms, int splits_override, bool pdl, unsigned long long timeout_ns,
                        cudaStream_t stream, GemmPlan* used) {
  if (M <= 0 || M > 256 || N <= 0 || K <= 0 || K % 8 || (dtype != kBF16 && dtype != kF16))
    return cudaErrorInvalidValue;
  const GemmPlan p = plan_gemm(M, N, K, num_sms, splits_override);
  if (used) *used = p;
  const bool bf16 = dtype == kBF16;
  CUtensorMap mw, mx;
  cudaError_t e = tensor_map(W, N, K, BM, bf16, &mw);
  if (e != cudaSuccess) return e;
  e = tensor_map(X, M, K, p.bn, bf16, &mx);
  if (e != cudaSuccess) return e;
  return bf16 ? launch_typed<true>(mw, mx, p.bn, Y, M, N, K, p.kps, p.splits, ldy, err, timeout_ns, pdl, stream)
              : launch_typed<false>(mw, mx, p.bn, Y, M, N, K, p.kps, p.splits, ldy, err, timeout_ns, pdl, stream);
}

}  // namespace cob
