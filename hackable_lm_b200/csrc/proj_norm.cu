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
// 4-byte store into (possibly another CTA's) shared memory that signals its
// completion as 4 transaction bytes on the mbarrier at `bar_cluster` in the same CTA
// as the destination: no fence or separate arrive is needed for the receiver to see it.
HLM_DEVICE void st_async_f32(uint32_t cluster_addr, float v, uint32_t bar_cluster) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(cluster_addr),
               "r"(__float_as_uint(v)), "r"(bar_cluster)
               : "memory");
}
// Prefetch a 2-D TMA box into L2 (no shared memory, no completion to wait for).
HLM_DEVICE float ld_shared_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Eight epilogue warps: two per TMEM lane quadrant, each taking every other
// 64-column group of its 32 rows, so the epilogue of a tile (residual wait, two
// passes, stores) stays shorter than the next tile's K loop.
constexpr int kProjNormEpiWarps = 8;
constexpr int kProjNormParts = kProjNormEpiWarps / 4;

template <int CL>
struct EpiResidualNorm {
  static_assert(CL >= 1 && CL <= 4, "1 to 4 CTAs per row block");
  static constexpr bool kClusterExchange = CL > 1;
  static constexpr int P = kProjNormParts;
  struct Params {
    alignas(64) CUtensorMap map_out;   // out  [M][N] bf16, box {64, 32}
    alignas(64) CUtensorMap map_norm;  // norm [M][N] bf16, box {64, 32}
    alignas(64) CUtensorMap map_res;   // residual [M][N] bf16, box {64, 32}
    int N;
    float eps;
  };
  static constexpr int kBoxBytes = 32 * 128;  // 32 rows x 64 bf16, 128-byte swizzle
  // Each epilogue warp owns the boxes of its 64-column groups (its 32 rows x 64
  // columns each, the TMA 128-byte-swizzle layout): the residual lands there by TMA,
  // pass 1 overwrites it in place with `out` and stores it, pass 2 writes `norm`
  // there and stores it.  A whole pass is staged before its stores drain, so they
  // run back to back.
  // Layout: [exchange mbarriers x2 | residual mbarriers x8 | sums float[2][CL][P][128] |
  //          pad to 1 KB | boxes].
  static constexpr int kBarsOffset = 0;
  static constexpr int kResBarsOffset = 16;
  static constexpr int kSumsOffset = 128;
  static constexpr int kStagingOffset = ((kSumsOffset + 2 * CL * P * kBM * 4 + 1023) / 1024) * 1024;
  template <int EPI_WARPS>
  static constexpr int smem_bytes() {
    static_assert(EPI_WARPS == kProjNormEpiWarps, "two epilogue warps per TMEM lane quadrant");
    return kStagingOffset + 4 * 4 * kBoxBytes;  // 4 lane quadrants x up to BN = 256 columns
  }
  static HLM_DEVICE void init(uint8_t* epi_smem) {
    const uint32_t bars = smem_u32(epi_smem) + kBarsOffset;
    mbar_init(bars, CL * P * kBM);  // one arrival per epilogue thread of every CTA
    mbar_init(bars + 8, CL * P * kBM);
    for (int w = 0; w < kProjNormEpiWarps; ++w)
      mbar_init(smem_u32(epi_smem) + kResBarsOffset + 8u * w, 1);  // the warp's residual loads
  }

  static HLM_DEVICE float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

  // 16-byte chunk c (8 columns) of a 64-column group, 4 packed bf16x2 words, into
  // a 32 x 64 box (128-byte swizzle: chunk index ^ row % 8)
  static HLM_DEVICE void stage_chunk(uint32_t box, int c, int lane, uint32_t w0, uint32_t w1, uint32_t w2,
                                     uint32_t w3) {
    st_shared_v4(box + static_cast<uint32_t>(lane * 128 + ((c ^ (lane & 7)) << 4)), make_uint4(w0, w1, w2, w3));
  }

  // One thread owns one row of the tile and the 64-column groups g = part, part + 2, ...
  // The warp's residual boxes arrive by TMA (coalesced, no load instructions); pass 1
  // keeps `out` in registers of packed bf16 pairs, which pass 2 scales, so neither the
  // accumulator nor the residual is read twice.
  template <int BN, int kParts>
  static HLM_DEVICE void run(const Params& ep, const GemmParams& p, uint8_t* smem, uint32_t taddr,
                             int m_tile, int n_tile, int, int quad, int part, int lane) {
    static_assert(kParts == P, "two epilogue warps per lane quadrant");
    static_assert(BN % (64 * P) == 0 && BN <= 256, "64-column store boxes, split over the parts");
    constexpr int GW = BN / 64 / P;  // groups of this warp
    // tile counter of this CTA (work index w = blockIdx.x + it * gridDim.x)
    const int it = (m_tile * p.n_tiles + n_tile - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x);
    const int b = it & 1;
    const uint32_t par = static_cast<uint32_t>((it >> 1) & 1);
    const int row_in = quad * 32 + lane;
    const int col0 = n_tile * BN;
    const int row0 = m_tile * kBM + quad * 32;
    const int wid = part * 4 + quad;
    const uint32_t base = smem_u32(smem);
    const uint32_t boxes = base + static_cast<uint32_t>(kStagingOffset + wid * GW * kBoxBytes);
    const uint32_t sums = base + kSumsOffset;
    const uint32_t bar = base + kBarsOffset + 8u * static_cast<uint32_t>(b);
    const uint32_t res_bar = base + kResBarsOffset + 8u * static_cast<uint32_t>(wid);

    // residual rows -> the warp's boxes (rows past M read as zero)
    if (lane == 0) {
      bulk_wait_group_read<0>();  // the previous tile's stores have read the boxes
      mbar_arrive_expect_tx(res_bar, static_cast<uint32_t>(GW * kBoxBytes));
#pragma unroll
      for (int i = 0; i < GW; ++i)
        tma_load_2d(boxes + static_cast<uint32_t>(i * kBoxBytes), &ep.map_res, col0 + (i * P + part) * 64, row0,
                    res_bar);
    }
    warp_wait(res_bar, static_cast<uint32_t>(it & 1), p.err, kDevErrTimeoutEpiLoad, lane);

    // ---- pass 1: out = bf16(bf16(acc) + residual), sum of squares, store out
    uint32_t pk[GW * 32];  // word 32 i + j = columns 2j, 2j+1 of this warp's group i
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < GW; ++i) {
      const int g = i * P + part;
      const uint32_t box = boxes + static_cast<uint32_t>(i * kBoxBytes);
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
            const float o0 = bf16r(bf16r(__uint_as_float(r[2 * j])) + bf16_lo(rw[k]));
            const float o1 = bf16r(bf16r(__uint_as_float(r[2 * j + 1])) + bf16_hi(rw[k]));
            ss = fmaf(o0, o0, ss);
            ss = fmaf(o1, o1, ss);
            pk[i * 32 + h * 16 + j] = pack_bf16x2(o0, o1);
          }
        }
      }
      // out over the residual, in place (each thread rewrites only its own row)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        stage_chunk(box, c, lane, pk[i * 32 + 4 * c], pk[i * 32 + 4 * c + 1], pk[i * 32 + 4 * c + 2],
                    pk[i * 32 + 4 * c + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&ep.map_out, col0 + g * 64, row0, box);
        bulk_commit_group();
      }
    }

    // ---- exchange this warp's partial row sum with every CTA of the cluster
    const uint32_t rank = CL > 1 ? cluster_ctarank() : 0u;
    const uint32_t slot =
        sums + static_cast<uint32_t>((((b * CL + static_cast<int>(rank)) * P + part) * kBM + row_in) * 4);
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
    for (int j = 0; j < CL * P; ++j) tot += ld_shared_f32(sums + static_cast<uint32_t>(((b * CL * P + j) * kBM + row_in) * 4));
    const float rstd = rsqrtf(tot / static_cast<float>(ep.N) + ep.eps);

    // ---- pass 2: norm = bf16(out * rstd)
    if (lane == 0) bulk_wait_group_read<0>();  // pass 1's stores have read the boxes
    __syncwarp();
#pragma unroll
    for (int i = 0; i < GW; ++i) {
      const int g = i * P + part;
      const uint32_t box = boxes + static_cast<uint32_t>(i * kBoxBytes);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t x = pk[i * 32 + 4 * c + q];
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

// ---------------------------------------------------------------------------
// CTA-pair variant for N a multiple of 256: clusters of 2 * CL CTAs, i.e. CL
// tcgen05 cta_group::2 pairs.  Pair j of a cluster (CTAs 2j, 2j + 1) computes the
// 256 x 256 tile (rows of the cluster's 256-row block, columns 256 j ..) exactly as
// gemm_pair_kernel does (each CTA loads its 128 A rows and half of B, the even CTA
// issues M = 256 MMAs, each CTA drains its own 128 accumulator rows), and the
// epilogues of the CTAs holding the same 128 rows (ranks h, 2 + h, 4 + h, ...)
// exchange their row sums.  Per SM this halves the B operand traffic of the
// single-CTA form above.
// ---------------------------------------------------------------------------
template <int CL>
struct EpiResidualNormPair {
  static_assert(CL >= 1 && CL <= 4, "1 to 4 pairs per row block");
  static constexpr int P = kProjNormParts;
  using Params = typename EpiResidualNorm<CL>::Params;
  static constexpr int kBoxBytes = EpiResidualNorm<CL>::kBoxBytes;
  static constexpr int kBarsOffset = 0;
  static constexpr int kResBarsOffset = 16;
  static constexpr int kSumsOffset = 128;
  static constexpr int kStagingOffset = ((kSumsOffset + 2 * CL * P * kBM * 4 + 1023) / 1024) * 1024;
  template <int EPI_WARPS>
  static constexpr int smem_bytes() {
    static_assert(EPI_WARPS == kProjNormEpiWarps, "two epilogue warps per TMEM lane quadrant");
    return kStagingOffset + 4 * 4 * kBoxBytes;
  }
  // Exchange barriers: one local arrival per tile (which also announces the bytes
  // to expect) and CL * P * 128 four-byte st.async transactions from the CTAs with
  // these rows, this one included.
  static constexpr uint32_t kExchangeBytes = CL * P * kBM * 4;
  static HLM_DEVICE void init(uint8_t* epi_smem) {
    const uint32_t bars = smem_u32(epi_smem) + kBarsOffset;
    mbar_init(bars, 1);
    mbar_init(bars + 8, 1);
    for (int w = 0; w < kProjNormEpiWarps; ++w) mbar_init(smem_u32(epi_smem) + kResBarsOffset + 8u * w, 1);
  }

  // Same two passes as EpiResidualNorm; `it` is this cluster's tile counter, `pair`
  // the pair index (= column tile), `half` which 128 rows of the pair tile this CTA holds.
  static HLM_DEVICE void run(const Params& ep, const GemmParams& p, uint8_t* smem, uint32_t taddr, int it,
                             int m_tile, int pair, int half, int quad, int part, int lane) {
    constexpr int BN = 256;
    constexpr int GW = BN / 64 / P;
    const int b = it & 1;
    const uint32_t par = static_cast<uint32_t>((it >> 1) & 1);
    const int row_in = quad * 32 + lane;
    const int col0 = pair * BN;
    const int row0 = m_tile * kBM + quad * 32;
    const int wid = part * 4 + quad;
    const uint32_t base = smem_u32(smem);
    const uint32_t boxes = base + static_cast<uint32_t>(kStagingOffset + wid * GW * kBoxBytes);
    const uint32_t sums = base + kSumsOffset;
    const uint32_t bar = base + kBarsOffset + 8u * static_cast<uint32_t>(b);
    const uint32_t res_bar = base + kResBarsOffset + 8u * static_cast<uint32_t>(wid);

    if (lane == 0) {
      bulk_wait_group_read<0>();
      mbar_arrive_expect_tx(res_bar, static_cast<uint32_t>(GW * kBoxBytes));
#pragma unroll
      for (int i = 0; i < GW; ++i)
        tma_load_2d(boxes + static_cast<uint32_t>(i * kBoxBytes), &ep.map_res, col0 + (i * P + part) * 64, row0,
                    res_bar);
      // the residual boxes of this warp's next tile, into L2 while this tile and the
      // next K loop run, so that tile's load above finds them there
      const int next_row0 = row0 + 2 * kBM * static_cast<int>(num_clusters_x());
      if (next_row0 < p.M) {
#pragma unroll
        for (int i = 0; i < GW; ++i) tma_prefetch_l2_2d(&ep.map_res, col0 + (i * P + part) * 64, next_row0);
      }
    }
    warp_wait(res_bar, static_cast<uint32_t>(it & 1), p.err, kDevErrTimeoutEpiLoad, lane);

    uint32_t pk[GW * 32];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < GW; ++i) {
      const int g = i * P + part;
      const uint32_t box = boxes + static_cast<uint32_t>(i * kBoxBytes);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(g * 64 + h * 32), r);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 rv = ld_shared_v4(box + static_cast<uint32_t>(lane * 128 + (((h * 4 + q) ^ (lane & 7)) << 4)));
          const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int j = q * 4 + k;
            const float o0 = EpiResidualNorm<CL>::bf16r(EpiResidualNorm<CL>::bf16r(__uint_as_float(r[2 * j])) +
                                                        bf16_lo(rw[k]));
            const float o1 = EpiResidualNorm<CL>::bf16r(EpiResidualNorm<CL>::bf16r(__uint_as_float(r[2 * j + 1])) +
                                                        bf16_hi(rw[k]));
            ss = fmaf(o0, o0, ss);
            ss = fmaf(o1, o1, ss);
            pk[i * 32 + h * 16 + j] = pack_bf16x2(o0, o1);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < 8; ++c)
        EpiResidualNorm<CL>::stage_chunk(box, c, lane, pk[i * 32 + 4 * c], pk[i * 32 + 4 * c + 1],
                                         pk[i * 32 + 4 * c + 2], pk[i * 32 + 4 * c + 3]);
    }
    fence_proxy_async_smem();  // one fence for the warp's whole pass
    __syncwarp();
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < GW; ++i)
        tma_store_2d(&ep.map_out, col0 + (i * P + part) * 64, row0, boxes + static_cast<uint32_t>(i * kBoxBytes));
      bulk_commit_group();
    }

    // the CTAs holding these rows: cluster ranks 2 j + half; each receives this
    // thread's partial by st.async, counted as transaction bytes on its barrier
    if (wid == 0 && lane == 0) mbar_arrive_expect_tx(bar, kExchangeBytes);
    const uint32_t slot = sums + static_cast<uint32_t>((((b * CL + pair) * P + part) * kBM + row_in) * 4);
#pragma unroll
    for (int j = 0; j < CL; ++j) {
      const uint32_t dst = static_cast<uint32_t>(2 * j + half);
      st_async_f32(mapa_shared(slot, dst), ss, mapa_shared(bar, dst));
    }
    mbar_wait_cluster(bar, par, p.err, kDevErrTimeoutPeer);
    float tot = 0.0f;
#pragma unroll
    for (int j = 0; j < CL * P; ++j)
      tot += ld_shared_f32(sums + static_cast<uint32_t>(((b * CL * P + j) * kBM + row_in) * 4));
    const float rstd = rsqrtf(tot / static_cast<float>(ep.N) + ep.eps);

    if (lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
#pragma unroll
    for (int i = 0; i < GW; ++i) {
      const uint32_t box = boxes + static_cast<uint32_t>(i * kBoxBytes);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t x = pk[i * 32 + 4 * c + q];
          w[q] = pack_bf16x2(bf16_lo(x) * rstd, bf16_hi(x) * rstd);
        }
        EpiResidualNorm<CL>::stage_chunk(box, c, lane, w[0], w[1], w[2], w[3]);
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < GW; ++i)
        tma_store_2d(&ep.map_norm, col0 + (i * P + part) * 64, row0, boxes + static_cast<uint32_t>(i * kBoxBytes));
      bulk_commit_group();
    }
  }
};

constexpr int kPairRowsStages = 4;  // 32 KB stages (16 KB of A + half of a 256-row B)

template <int CL>
__global__ void __launch_bounds__(gemm_threads<kProjNormEpiWarps>(), 1)
    gemm_pair_rows_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const GemmParams p, const __grid_constant__ typename EpiResidualNorm<CL>::Params ep) {
  constexpr int BN = 256;
  constexpr int STAGES = kPairRowsStages;
  constexpr int EPI_WARPS = kProjNormEpiWarps;
  using L = PairSmem<BN, STAGES>;
  using Epi = EpiResidualNormPair<CL>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t half = rank & 1u;       // which 128 rows of the pair tile
  const uint32_t even = rank & ~1u;      // the pair's MMA-issuing CTA
  const int pair = static_cast<int>(rank >> 1);  // column tile of this pair
  const uint32_t bar0 = base + L::kBarOffset;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + L::kTmemSlotOffset);
  int* err = p.err;
#define FULL_BAR(s) (bar0 + 8u * (s))
#define EMPTY_BAR(s) (bar0 + 8u * (STAGES + (s)))
#define TFULL_BAR(a) (bar0 + 8u * (2 * STAGES + (a)))
#define TEMPTY_BAR(a) (bar0 + 8u * (2 * STAGES + 2 + (a)))

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(FULL_BAR(s), 1);
      mbar_init(EMPTY_BAR(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(TFULL_BAR(a), 1);
      mbar_init(TEMPTY_BAR(a), 2 * EPI_WARPS);
    }
    Epi::init(base_ptr + L::kEpiOffset);
    fence_mbar_init();
    prefetch_tensormap(&tmA);
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const int m_pairs = p.m_tiles;  // 256-row blocks
  const int c_first = static_cast<int>(cluster_id_x());
  const int c_step = static_cast<int>(num_clusters_x());

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_mask = 0, armed_par = 0;
      bool ok = true;
      const uint32_t sb_off = L::kABytes;
      for (int mp = c_first; mp < m_pairs && ok; mp += c_step) {
        const int m0 = (2 * mp + static_cast<int>(half)) * kBM;
        const int nb0 = pair * BN + static_cast<int>(half) * (BN / 2);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(EMPTY_BAR(stage), phase ^ 1u, err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (half == 0) {
            mbar_arrive_expect_tx(FULL_BAR(stage), 2 * L::kStageBytes);
            armed_mask |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t full = mapa_shared(FULL_BAR(stage), even);
          const uint32_t sa = base + stage * L::kStageBytes;
          const int k0 = kb * kBK;
          tma_load_2d_pair(sa, &tmA, k0, m0, full);
#pragma unroll
          for (int i = 0; i < BN / 128; ++i) tma_load_2d_pair(sa + sb_off + i * 8192u, &tmB, k0, nb0 + 64 * i, full);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < STAGES; ++s)
        if (armed_mask & (1u << s)) mbar_wait_drain(FULL_BAR(s), (armed_par >> s) & 1u, err);
    }
  } else if (warp == 1) {
    if (lane == 0 && half == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(2 * kBM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int mp = c_first; mp < m_pairs && ok; mp += c_step, ++it) {
        const int acc = it & 1;
        const uint32_t acc_par = static_cast<uint32_t>((it >> 1) & 1);
        if (!mbar_wait_cluster(TEMPTY_BAR(acc), acc_par ^ 1u, err, kDevErrTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_cluster(FULL_BAR(stage), phase, err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk)
            tc_mma_f16_pair(d_tmem, make_sw128_desc(sa + kk * 32u, 16u, 1024u),
                            make_sw128_desc(sb + kk * 32u, 16u, 1024u), idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          tc_commit_pair(EMPTY_BAR(stage));
          tc_commit_pair(mapa_shared(EMPTY_BAR(stage), even | 1u));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(TFULL_BAR(acc));
        tc_commit_pair(mapa_shared(TFULL_BAR(acc), even | 1u));
      }
    }
  } else {
    const int quad = warp & 3;
    const int part = (warp - kEpiWarp0) >> 2;
    int it = 0;
    for (int mp = c_first; mp < m_pairs; mp += c_step, ++it) {
      const int acc = it & 1;
      const uint32_t acc_par = static_cast<uint32_t>((it >> 1) & 1);
      if (!warp_wait(TFULL_BAR(acc), acc_par, err, kDevErrTimeoutTmemFull, lane)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      Epi::run(ep, p, base_ptr + L::kEpiOffset, taddr, it, 2 * mp + static_cast<int>(half), pair,
               static_cast<int>(half), quad, part, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(TEMPTY_BAR(acc), even));
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncwarp();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, L::kTmemCols);
  }
#undef FULL_BAR
#undef EMPTY_BAR
#undef TFULL_BAR
#undef TEMPTY_BAR
}

template <int CL>
static int launch_pair_rows(const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p,
                            const typename EpiResidualNorm<CL>::Params& ep, cudaStream_t s) {
  using L = PairSmem<256, kPairRowsStages>;
  auto kern = gemm_pair_rows_kernel<CL>;
  constexpr int smem = L::kEpiOffset + EpiResidualNormPair<CL>::template smem_bytes<kProjNormEpiWarps>() + 1024;
  static_assert(smem <= 232448, "shared memory budget exceeded");
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  if (2 * CL > 8 && cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  if (p.m_tiles <= 0) return HLM_OK;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(2 * CL);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(gemm_threads<kProjNormEpiWarps>(), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = num_sms_of_current_device() / (2 * CL);
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * 2 * CL), 1, 1);
  int fit = 0;
  if (cudaOccupancyMaxActiveClusters(&fit, kern, &cfg) == cudaSuccess && fit > 0 && fit < clusters) clusters = fit;
  if (clusters > p.m_tiles) clusters = p.m_tiles;
  if (clusters < 1) clusters = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * 2 * CL), 1, 1);
  {
    LaunchScope scope(HLM_KERNEL_PROJ_NORM, s);
    if (cudaLaunchKernelEx(&cfg, kern, ma, mb, p, ep) != cudaSuccess) return HLM_ERR_LAUNCH;
  }
  return launch_status();
}

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

static int proj_norm_pair_dispatch(int cl, const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p,
                                   const CUtensorMap& mo, const CUtensorMap& mn, const CUtensorMap& mr, int N,
                                   float eps, cudaStream_t s) {
#define HLM_PNP_CASE(CLV)                                                    \
  case CLV: {                                                                \
    typename EpiResidualNorm<CLV>::Params ep;                                \
    ep.map_out = mo;                                                         \
    ep.map_norm = mn;                                                        \
    ep.map_res = mr;                                                         \
    ep.N = N;                                                                \
    ep.eps = eps;                                                            \
    return launch_pair_rows<CLV>(ma, mb, p, ep, s);                          \
  }
  switch (cl) {
    HLM_PNP_CASE(1)
    HLM_PNP_CASE(2)
    HLM_PNP_CASE(3)
    HLM_PNP_CASE(4)
    default:
      return HLM_ERR_UNSUPPORTED;
  }
#undef HLM_PNP_CASE
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
  // B boxes: 64 rows for the CTA-pair kernel (each CTA loads half of a 256-row tile),
  // the whole BN-row tile for the single-CTA kernel
  if (!encode_bf16_map(&ma, y, K, M, K, kBM) || !encode_bf16_map(&mb, w, K, N, K, bn == 256 ? 64 : bn) ||
      !encode_bf16_map(&mo, out, N, M, N, 32) || !encode_bf16_map(&mn, norm, N, M, N, 32) ||
      !encode_bf16_map(&mr, residual, N, M, N, 32))
    return HLM_ERR_DRIVER;
  GemmParams p;
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (bn == 256) {
    gemm_tiling_pair(p, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), 256, 1);
    return proj_norm_pair_dispatch(cl, ma, mb, p, mo, mn, mr, static_cast<int>(N), eps, s);
  }
  gemm_tiling(p, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), bn, 1);
  return proj_norm_dispatch<128>(cl, ma, mb, p, mo, mn, mr, static_cast<int>(N), eps, s);
}
