// Host side of the tcgen05 GEMM core: tensor-map encoding through the driver
// entry point (no link-time dependency on libcuda) and the plain GEMM entry
// point.
#include <mutex>

#include "gemm_sm100.cuh"

namespace hlm {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

bool encode_bf16_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t ld, uint32_t box_outer) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return false;
  if (!host_aligned16(base) || (ld % 8) != 0 || inner == 0 || outer == 0 || ld < inner) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r =
      fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, bool A_MN, bool B_MN>
static int plain_gemm(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K,
                      int64_t lda, int64_t ldb, int64_t ldd, int d_dtype, int accumulate,
                      cudaStream_t s) {
  constexpr int STAGES = BN == 256 ? 4 : 6;
  CUtensorMap ma, mb;
  bool ok = A_MN ? encode_bf16_map(&ma, A, M, K, lda, 64) : encode_bf16_map(&ma, A, K, M, lda, kBM);
  ok = ok && (B_MN ? encode_bf16_map(&mb, B, N, K, ldb, 64) : encode_bf16_map(&mb, B, K, N, ldb, BN));
  if (!ok) return HLM_ERR_DRIVER;
  GemmParams p;
  gemm_tiling(p, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), BN, 1);
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  EpiStore::Params ep;
  ep.d = D;
  ep.ldd = ldd;
  ep.split_stride = 0;
  ep.dtype = d_dtype;
  ep.accumulate = accumulate;
  const int esz = d_dtype == HLM_F32 ? 4 : 2;
  ep.vec_ok = host_aligned16(D) && ((ldd * esz) % 16 == 0);
  ep.alpha = nullptr;
  return launch_gemm_sm100<BN, STAGES, A_MN, B_MN, EpiStore>(ma, ma, ma, mb, p, ep, s,
                                                              HLM_KERNEL_GEMM);
}

// CTA-pair version (M >= 256): 256 x BN tiles, each CTA loads half of B.
template <int BN, bool A_MN, bool B_MN>
static int plain_gemm_pair(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K,
                           int64_t lda, int64_t ldb, int64_t ldd, int d_dtype, int accumulate,
                           cudaStream_t s) {
  constexpr int STAGES = BN == 384 ? 5 : (BN == 256 ? 6 : 8);
  CUtensorMap ma, mb;
  bool ok = A_MN ? encode_bf16_map(&ma, A, M, K, lda, 64) : encode_bf16_map(&ma, A, K, M, lda, kBM);
  ok = ok && (B_MN ? encode_bf16_map(&mb, B, N, K, ldb, 64) : encode_bf16_map(&mb, B, K, N, ldb, 64));
  if (!ok) return HLM_ERR_DRIVER;
  GemmParams p;
  gemm_tiling_pair(p, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), BN, 1);
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  EpiStore::Params ep;
  ep.d = D;
  ep.ldd = ldd;
  ep.split_stride = 0;
  ep.dtype = d_dtype;
  ep.accumulate = accumulate;
  const int esz = d_dtype == HLM_F32 ? 4 : 2;
  ep.vec_ok = host_aligned16(D) && ((ldd * esz) % 16 == 0);
  ep.alpha = nullptr;
  return launch_gemm_pair<BN, STAGES, A_MN, B_MN, EpiStore>(ma, ma, ma, mb, p, ep, s, HLM_KERNEL_GEMM);
}

}  // namespace hlm

using namespace hlm;

extern "C" int hlm_gemm_bf16(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K,
                             int a_mn_major, int b_mn_major, int64_t lda, int64_t ldb, int64_t ldd,
                             int d_dtype, int accumulate, void* stream) {
  if (M < 0 || N < 0 || K < 0) return HLM_ERR_INVALID_ARG;
  if (M == 0 || N == 0) return HLM_OK;
  if (A == nullptr || B == nullptr || D == nullptr) return HLM_ERR_INVALID_ARG;
  if (d_dtype != HLM_BF16 && d_dtype != HLM_F32) return HLM_ERR_UNSUPPORTED;
  if (M > (1ll << 31) - 256 || N > (1ll << 31) - 256 || K > (1ll << 31) - 256)
    return HLM_ERR_UNSUPPORTED;
  if (ldd < N) return HLM_ERR_INVALID_ARG;
  if (K == 0) return HLM_ERR_UNSUPPORTED;  // an empty reduction is not a tensor-core job
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool wide = N > 128;
  const int am = a_mn_major ? 1 : 0, bm = b_mn_major ? 1 : 0;
#define HLM_PAIR(BNV, AM, BM)                                                                  \
  return plain_gemm_pair<BNV, AM, BM>(A, B, D, M, N, K, lda, ldb, ldd, d_dtype, accumulate, s)
  if (M >= 2 * kBM) {
    if (N % 384 == 0 && K >= 8192) {
      // long K: 256 x 384 pair tiles (one accumulator, whose epilogue is then a
      // small share of the tile), less B traffic per FLOP
      if (!am && !bm) HLM_PAIR(384, false, false);
      if (!am && bm) HLM_PAIR(384, false, true);
      if (am && !bm) HLM_PAIR(384, true, false);
      HLM_PAIR(384, true, true);
    }
    if (wide) {
      if (!am && !bm) HLM_PAIR(256, false, false);
      if (!am && bm) HLM_PAIR(256, false, true);
      if (am && !bm) HLM_PAIR(256, true, false);
      HLM_PAIR(256, true, true);
    } else {
      if (!am && !bm) HLM_PAIR(128, false, false);
      if (!am && bm) HLM_PAIR(128, false, true);
      if (am && !bm) HLM_PAIR(128, true, false);
      HLM_PAIR(128, true, true);
    }
  }
#undef HLM_PAIR
#define HLM_PLAIN(BNV, AM, BM)                                                                 \
  return plain_gemm<BNV, AM, BM>(A, B, D, M, N, K, lda, ldb, ldd, d_dtype, accumulate, s)
  if (wide) {
    if (!am && !bm) HLM_PLAIN(256, false, false);
    if (!am && bm) HLM_PLAIN(256, false, true);
    if (am && !bm) HLM_PLAIN(256, true, false);
    HLM_PLAIN(256, true, true);
  } else {
    if (!am && !bm) HLM_PLAIN(128, false, false);
    if (!am && bm) HLM_PLAIN(128, false, true);
    if (am && !bm) HLM_PLAIN(128, true, false);
    HLM_PLAIN(128, true, true);
  }
#undef HLM_PLAIN
}
