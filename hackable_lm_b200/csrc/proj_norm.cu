// Output / down projection with the residual add and the weightless RMSNorm
// of the next sublayer's input in the GEMM epilogue.
//
//   branch = bf16(y @ w^T)          the nn.Linear output (model.py:261-264, 303-304)
//   out    = bf16(residual + branch)  the next residual stream (model.py:73-74)
//   norm   = bf16(out * rsqrt(mean(out^2) + eps))        (model.py:14-16, 75)
//
// The RMS needs the whole row of N (768 at d12) outputs, wider than one TMEM
// accumulator pair allows.  So the single-CTA tcgen05 GEMM core runs in
// thread-block clusters of CL = N / BN CTAs: the CTAs of a cluster take the CL
// column tiles of the same 128-row block (each loads the same A rows and its own
// BN rows of w; no load is multicast), and their epilogues exchange per-row sums
// of squares through distributed shared memory:
//
//   pass 1  read the accumulator chunk by chunk, round to bf16, add the residual
//           (loaded for the whole row at the start of the tile), round, keep `out`
//           in registers, store it (TMA, 32x64 boxes) and sum the squares;
//   swap    write the row's partial sum into slot [buf][rank][row] of every CTA of
//           the cluster (st.shared::cluster) and arrive on each CTA's mbarrier
//           (release, cluster scope); wait on this CTA's barrier (acquire), add
//           the CL partials;
//   pass 2  scale the kept `out` by 1/rms, store `norm`.
//
// Two slot buffers / barriers alternate by tile, so a CTA can be at most one tile
// ahead of a peer (it cannot finish tile i+1 before receiving the peer's tile i+1
// partial, sent after the peer has read tile i's).  Every wait is bounded.
// With two TMEM accumulators (2 x BN <= 512 columns) the epilogue of tile i
// overlaps the MMAs of tile i+1.
#include "gemm_sm100.cuh"

namespace hlm {

HLM_DEVICE void st_shared_cluster_f32(uint32_t cluster_addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(cluster_addr), "f"(v) : "memory");
}
HLM_DEVICE float ld_shared_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

constexpr int kProjNormEpiWarps = 4;

template <int CL>
struct EpiResidualNorm {
  static_assert(CL >= 1 && CL <= 4, "1 to 4 CTAs per row block");
  static constexpr bool kClusterExchange = CL > 1;
  struct Params {
    alignas(64) CUtensorMap map_out;   // out  [M][N] bf16, box {64, 32}
    alignas(64) CUtensorMap map_norm;  // norm [M][N] bf16, box {64, 32}
    alignas(64) CUtensorMap map_res;   // residual [M][N] bf16, box {64, 32}
    int N;
    float eps;
  };
  static constexpr int kBoxBytes = 32 * 128;  // 32 rows x 64 bf16, 128-byte swizzle
  // Each epilogue warp owns BN / 64 boxes (its 32 rows x 64 columns each, the TMA
  // 128-byte-swizzle layout): the residual lands there by TMA, pass 1 overwrites it
  // in place with `out` and stores it, pass 2 writes `norm` there and stores it.  A
  // whole pass is staged before its stores drain, so they run back to back.
  // Layout: [exchange mbarriers x2 | residual mbarriers x4 | sums float[2][CL][128] |
  //          pad to 1 KB | boxes].
  static constexpr int kBarsOffset = 0;
  static constexpr int kResBarsOffset = 16;
  static constexpr int kSumsOffset = 48;
  static constexpr int kStagingOffset = ((kSumsOffset + 2 * CL * kBM * 4 + 1023) / 1024) * 1024;
  template <int EPI_WARPS>
  static constexpr int smem_bytes() {
    static_assert(EPI_WARPS == kProjNormEpiWarps, "one epilogue warp per TMEM lane quadrant");
    return kStagingOffset + kProjNormEpiWarps * 4 * kBoxBytes;  // up to BN = 256 per warp
  }
  static HLM_DEVICE void init(uint8_t* epi_smem) {
    const uint32_t bars = smem_u32(epi_smem) + kBarsOffset;
    mbar_init(bars, CL * kBM);  // one arrival per epilogue thread of every CTA
    mbar_init(bars + 8, CL * kBM);
    for (int w = 0; w < kProjNormEpiWarps; ++w)
      mbar_init(smem_u32(epi_smem) + kResBarsOffset + 8u * w, 1);  // the warp's residual loads
  }

  static HLM_DEVICE float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

  // 16-byte chunk c (8 columns) of a 64-column group, 4 packed bf16x2 words, into
  // the warp's 32 x 64 staging box (128-byte swizzle: chunk index ^ row % 8)
  static HLM_DEVICE void stage_chunk(uint32_t box, int c, int lane, uint32_t w0, uint32_t w1, uint32_t w2,
                                     uint32_t w3) {
    st_shared_v4(box + static_cast<uint32_t>(lane * 128 + ((c ^ (lane & 7)) << 4)), make_uint4(w0, w1, w2, w3));
  }

  // One thread owns one row of the tile.  The warp's residual rows arrive by TMA (one
  // load per 64-column box, coalesced, no load instructions); pass 1 keeps `out` in
  // BN / 2 registers of packed bf16 pairs, which pass 2 scales, so neither the
  // accumulator nor the residual is read twice.
  template <int BN, int kParts>
  static HLM_DEVICE void run(const Params& ep, const GemmParams& p, uint8_t* smem, uint32_t taddr,
                             int m_tile, int n_tile, int, int quad, int, int lane) {
    static_assert(kParts == 1, "four epilogue warps");
    static_assert(BN % 64 == 0, "64-column store boxes");
    constexpr int G = BN / 64;  // 64-column groups
    // tile counter of this CTA (work index w = blockIdx.x + it * gridDim.x)
    const int it = (m_tile * p.n_tiles + n_tile - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x);
    const int b = it & 1;
    const uint32_t par = static_cast<uint32_t>((it >> 1) & 1);
    const int row_in = quad * 32 + lane;
    const int row = m_tile * kBM + row_in;
    const bool row_ok = row < p.M;
    const int col0 = n_tile * BN;
    const int row0 = m_tile * kBM + quad * 32;
    (void)row_ok;
    static_assert(BN <= 256, "staging holds up to four 64-column boxes per warp");
    const uint32_t base = smem_u32(smem);
    const uint32_t boxes = base + static_cast<uint32_t>(kStagingOffset + quad * G * kBoxBytes);
    const uint32_t sums = base + kSumsOffset;
    const uint32_t bar = base + kBarsOffset + 8u * static_cast<uint32_t>(b);
    const uint32_t res_bar = base + kResBarsOffset + 8u * static_cast<uint32_t>(quad);

    // residual rows -> the warp's boxes (rows past M read as zero)
    if (lane == 0) {
      bulk_wait_group_read<0>();  // the previous tile's stores have read the boxes
      mbar_arrive_expect_tx(res_bar, static_cast<uint32_t>(G * kBoxBytes));
#pragma unroll
      for (int g = 0; g < G; ++g)
        tma_load_2d(boxes + static_cast<uint32_t>(g * kBoxBytes), &ep.map_res, col0 + g * 64, row0, res_bar);
    }
    warp_wait(res_bar, static_cast<uint32_t>(it & 1), p.err, kDevErrTimeoutEpiLoad, lane);

    // ---- pass 1: out = bf16(bf16(acc) + residual), sum of squares, store out
    uint32_t pk[BN / 2];  // word i = columns 2i, 2i+1 of `out`
    float ss = 0.0f;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint32_t box = boxes + static_cast<uint32_t>(g * kBoxBytes);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(g * 64 + h * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {  // 16-byte chunk h * 4 + q of the box row
          const uint4 rv = ld_shared_v4(box + static_cast<uint32_t>(lane * 128 + (((h * 4 + q) ^ (lane & 7)) << 4)));
          const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int j = q * 4 + k;  // word within the 32-column half
            const int wi = g * 32 + h * 16 + j;
            const float o0 = bf16r(bf16r(__uint_as_float(r[2 * j])) + bf16_lo(rw[k]));
            const float o1 = bf16r(bf16r(__uint_as_float(r[2 * j + 1])) + bf16_hi(rw[k]));
            ss = fmaf(o0, o0, ss);
            ss = fmaf(o1, o1, ss);
            pk[wi] = pack_bf16x2(o0, o1);
          }
        }
      }
      // out over the residual, in place (each thread rewrites only its own row)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        stage_chunk(box, c, lane, pk[g * 32 + 4 * c], pk[g * 32 + 4 * c + 1], pk[g * 32 + 4 * c + 2],
                    pk[g * 32 + 4 * c + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&ep.map_out, col0 + g * 64, row0, box);
        bulk_commit_group();
      }
    }

    // ---- exchange the row's partial sum with every CTA of the cluster
    const uint32_t rank = CL > 1 ? cluster_ctarank() : 0u;
    const uint32_t slot = sums + static_cast<uint32_t>(((b * CL + static_cast<int>(rank)) * kBM + row_in) * 4);
#pragma unroll
    for (int j = 0; j < CL; ++j) {
      if constexpr (CL > 1) {
        st_shared_cluster_f32(mapa_shared(slot, static_cast<uint32_t>(j)), ss);
        mbar_arrive_cluster(mapa_shared(bar, static_cast<uint32_t>(j)));
      } else {
        st_shared_cluster_f32(slot, ss);
        mbar_arrive_cluster(bar);
      }
    }
    mbar_wait_cluster(bar, par, p.err, kDevErrTimeoutPeer);
    float tot = 0.0f;
#pragma unroll
    for (int j = 0; j < CL; ++j) tot += ld_shared_f32(sums + static_cast<uint32_t>(((b * CL + j) * kBM + row_in) * 4));
    const float rstd = rsqrtf(tot / static_cast<float>(ep.N) + ep.eps);

    // ---- pass 2: norm = bf16(out * rstd)
    if (lane == 0) bulk_wait_group_read<0>();  // pass 1's stores have read the boxes
    __syncwarp();
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const uint32_t box = boxes + static_cast<uint32_t>(g * kBoxBytes);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t x = pk[g * 32 + 4 * c + q];
          w[q] = pack_bf16x2(bf16_lo(x) * rstd, bf16_hi(x) * rstd);
        }
        stage_chunk(box, c, lane, w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&ep.map_norm, col0 + g * 64, row0, box);
        bulk_commit_group();
      }
    }
  }
};

template <int BN>
constexpr int proj_norm_stages() {
  return BN == 256 ? 3 : 4;  // 48 KB / 32 KB stages beside 64 KB of store staging
}

template <int BN, int CL>
static int proj_norm_launch(const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p,
                            const typename EpiResidualNorm<CL>::Params& ep, cudaStream_t s) {
  return launch_gemm_cluster<BN, proj_norm_stages<BN>(), false, false, EpiResidualNorm<CL>, kProjNormEpiWarps>(
      ma, ma, ma, mb, p, ep, CL, s, HLM_KERNEL_PROJ_NORM);
}

template <int BN>
static int proj_norm_dispatch(int cl, const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p,
                              const CUtensorMap& mo, const CUtensorMap& mn, const CUtensorMap& mr, int N,
                              float eps, cudaStream_t s) {
#define HLM_PN_CASE(CLV)                                                     \
  case CLV: {                                                                \
    typename EpiResidualNorm<CLV>::Params ep;                                \
    ep.map_out = mo;                                                         \
    ep.map_norm = mn;                                                        \
    ep.map_res = mr;                                                         \
    ep.N = N;                                                                \
    ep.eps = eps;                                                            \
    return proj_norm_launch<BN, CLV>(ma, mb, p, ep, s);                      \
  }
  switch (cl) {
    HLM_PN_CASE(1)
    HLM_PN_CASE(2)
    HLM_PN_CASE(3)
    HLM_PN_CASE(4)
    default:
      return HLM_ERR_UNSUPPORTED;
  }
#undef HLM_PN_CASE
}

}  // namespace hlm

using namespace hlm;

extern "C" int hlm_proj_residual_rms_norm_fwd(const void* y, const void* w, const void* residual, void* out,
                                              void* norm, int64_t M, int64_t K, int64_t N, float eps,
                                              void* stream) {
  if (M < 0 || K <= 0 || N <= 0) return HLM_ERR_INVALID_ARG;
  if (M == 0) return HLM_OK;
  if (y == nullptr || w == nullptr || residual == nullptr || out == nullptr || norm == nullptr)
    return HLM_ERR_INVALID_ARG;
  if (K % 64 != 0 || M > (1ll << 31) - 256) return HLM_ERR_UNSUPPORTED;
  int bn = 0;
  if (N % 256 == 0 && N / 256 <= 4)
    bn = 256;
  else if (N % 128 == 0 && N / 128 <= 4)
    bn = 128;
  else
    return HLM_ERR_UNSUPPORTED;
  const int cl = static_cast<int>(N / bn);
  const void* ptrs[] = {y, w, residual, out, norm};
  for (const void* ptr : ptrs)
    if (!host_aligned16(ptr)) return HLM_ERR_UNSUPPORTED;
  CUtensorMap ma, mb, mo, mn, mr;
  if (!encode_bf16_map(&ma, y, K, M, K, kBM) || !encode_bf16_map(&mb, w, K, N, K, bn) ||
      !encode_bf16_map(&mo, out, N, M, N, 32) || !encode_bf16_map(&mn, norm, N, M, N, 32) ||
      !encode_bf16_map(&mr, residual, N, M, N, 32))
    return HLM_ERR_DRIVER;
  GemmParams p;
  gemm_tiling(p, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), bn, 1);
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bn == 256)
    return proj_norm_dispatch<256>(cl, ma, mb, p, mo, mn, mr, static_cast<int>(N), eps, s);
  return proj_norm_dispatch<128>(cl, ma, mb, p, mo, mn, mr, static_cast<int>(N), eps, s);
}
