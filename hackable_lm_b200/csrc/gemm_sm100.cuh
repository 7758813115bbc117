// Persistent warp-specialised tcgen05 GEMM core for sm_100a.
//
//   D[M, N] (+)= A[M, K] * B[N, K]^T      bf16 operands, fp32 accumulation in TMEM
//
// Roles (one CTA per SM, grid = min(#tiles, #SMs)):
//   warp 0      : one thread issues TMA loads (cp.async.bulk.tensor, 128-byte
//                 swizzle) into a STAGES-deep shared-memory ring
//   warp 1      : allocates TMEM; one thread issues tcgen05.mma (M=128, N=BN,
//                 K=16) and tcgen05.commit to release stages / publish tiles
//   next EPI_WARPS warps (4 or 8): epilogue; warp w reads TMEM lanes
//                 32*(w%4)..+31 (one accumulator row per thread); with 8
//                 warps two warps share a lane quadrant and split its columns
// Two accumulators of BN columns each live in TMEM, so the epilogue of tile i
// overlaps the MMAs of tile i+1.
//
// Operand layouts: each operand is either K-major (stored [rows][ld], K
// contiguous; one TMA box {64, rows} per stage) or MN-major (stored [K][ld],
// M or N contiguous; rows/64 boxes {64, 64} per stage).  The contiguous
// dimension of A may be the concatenation of up to three tensors
// ("segments", boundaries a_seg1 / a_seg2), which lets the QKV backward read
// dq/dk/dv in place as one concatenated operand.
//
// Every mbarrier wait is bounded (see mbar_wait); on a timeout the kernel
// records an error code, drains its own in-flight TMA copies, frees TMEM and
// returns.
#pragma once

#include <type_traits>

#include "hlm_common.cuh"

namespace hlm {

// Epilogues may declare `static HLM_DEVICE void init(uint8_t* epi_smem)`: the
// kernel calls it from the thread that initialises the pipeline barriers,
// before the fence and the CTA/cluster barrier that publish them (for an
// epilogue's own mbarriers and counters in its shared-memory region).
template <class E, class = void>
struct epi_has_init : std::false_type {};
template <class E>
struct epi_has_init<E, std::void_t<decltype(E::init(static_cast<uint8_t*>(nullptr)))>> : std::true_type {};

// Epilogues of the single-CTA kernel that exchange data with the other CTAs of
// a thread-block cluster (launch_gemm_cluster) declare
// `static constexpr bool kClusterExchange = true`: the kernel then adds a
// cluster barrier after its barrier initialisation (no CTA signals a peer's
// barrier before the peer initialised it) and before it exits (no CTA leaves
// while a peer may still write its shared memory).
template <class E, class = void>
struct epi_cluster_exchange : std::false_type {};
template <class E>
struct epi_cluster_exchange<E, std::void_t<decltype(E::kClusterExchange)>>
    : std::integral_constant<bool, E::kClusterExchange> {};

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 bf16 = one 128-byte swizzle row
constexpr int kUmmaK = 16;
constexpr int kEpiWarp0 = 2;

template <int EPI_WARPS>
constexpr int gemm_threads() {
  return 32 * (2 + EPI_WARPS);
}

struct GemmParams {
  int M, N, K;
  int m_tiles, n_tiles, k_blocks;
  int splits, kb_per_split;
  // A's contiguous dimension may be the concatenation of three tensors:
  // [0, a_seg1) -> map 0, [a_seg1, a_seg2) -> map 1, [a_seg2, ...) -> map 2.
  // a_seg1 == 0 means a single tensor.  Boundaries are multiples of 64.
  int a_seg1, a_seg2;
  // Pair kernel, BN <= 256 only: when > 0, CTA r of a pair loads its half of B
  // from rows n_tile * BN/2 + r * b_pair_stride (two separate row ranges of B,
  // e.g. the gate and up halves of a packed gate/up weight) instead of the
  // contiguous n_tile * BN + r * BN/2.
  int b_pair_stride;
  int* err;
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kNumBars = 2 * STAGES + 4;
  static constexpr int kTmemSlotOffset = kBarOffset + kNumBars * 8;
  static constexpr int kEpiOffset = ((kTmemSlotOffset + 16 + 1023) / 1024) * 1024;
  static constexpr int kTmemCols = 2 * BN;
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation must be a power of two");
};

HLM_DEVICE void decode_work(int w, const GemmParams& p, int& m_tile, int& n_tile, int& split) {
  const int per_split = p.m_tiles * p.n_tiles;
  split = w / per_split;
  const int r = w - split * per_split;
  m_tile = r / p.n_tiles;
  n_tile = r - m_tile * p.n_tiles;
}

HLM_DEVICE void select_segment(const GemmParams& p, int& c, const CUtensorMap*& mp,
                               const CUtensorMap* m0, const CUtensorMap* m1,
                               const CUtensorMap* m2) {
  if (c < p.a_seg1) {
    mp = m0;
  } else if (c < p.a_seg2) {
    c -= p.a_seg1;
    mp = m1;
  } else {
    c -= p.a_seg2;
    mp = m2;
  }
}

// Wait that ignores the error word (used only to drain in-flight TMA copies
// before the CTA exits); bounded by the same timeout.
HLM_DEVICE bool mbar_wait_drain(uint32_t bar, uint32_t parity, int* err) {
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, kDevErrTimeoutDrain);
      return false;
    }
  }
  return true;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EPI_WARPS = 4>
__global__ void __launch_bounds__(gemm_threads<EPI_WARPS>(), 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA0,
                      const __grid_constant__ CUtensorMap tmA1,
                      const __grid_constant__ CUtensorMap tmA2,
                      const __grid_constant__ CUtensorMap tmB, const GemmParams p,
                      const __grid_constant__ typename Epi::Params ep) {
  using L = GemmSmem<BN, STAGES>;
  static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "4 or 8 epilogue warps");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
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
      mbar_init(TEMPTY_BAR(a), EPI_WARPS);  // one arrival per epilogue warp
    }
    if constexpr (epi_has_init<Epi>::value) Epi::init(base_ptr + L::kEpiOffset);
    fence_mbar_init();
    prefetch_tensormap(&tmA0);
    if (p.a_seg1 > 0) {
      prefetch_tensormap(&tmA1);
      prefetch_tensormap(&tmA2);
    }
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (epi_cluster_exchange<Epi>::value) cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  const int total = p.m_tiles * p.n_tiles * p.splits;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_mask = 0, armed_par = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x) {
        int m_tile, n_tile, split;
        decode_work(w, p, m_tile, n_tile, split);
        const int m0 = m_tile * kBM;
        const int n0 = n_tile * BN;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(EMPTY_BAR(stage), phase ^ 1u, err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(FULL_BAR(stage), L::kStageBytes);
          armed_mask |= 1u << stage;
          armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
          const int k0 = kb * kBK;
          // ---- A
          if constexpr (!A_MN) {
            const CUtensorMap* mp = &tmA0;
            int kc = k0;
            if (p.a_seg1 > 0) select_segment(p, kc, mp, &tmA0, &tmA1, &tmA2);
            tma_load_2d(sa, mp, kc, m0, FULL_BAR(stage));
          } else {
#pragma unroll
            for (int i = 0; i < kBM / 64; ++i) {
              const CUtensorMap* mp = &tmA0;
              int mc = m0 + 64 * i;
              if (p.a_seg1 > 0) select_segment(p, mc, mp, &tmA0, &tmA1, &tmA2);
              tma_load_2d(sa + i * 8192u, mp, mc, k0, FULL_BAR(stage));
            }
          }
          // ---- B
          if constexpr (!B_MN) {
            tma_load_2d(sb, &tmB, k0, n0, FULL_BAR(stage));
          } else {
#pragma unroll
            for (int i = 0; i < BN / 64; ++i) tma_load_2d(sb + i * 8192u, &tmB, n0 + 64 * i, k0, FULL_BAR(stage));
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain: every stage we armed must have landed before shared memory is
      // released (immediate in normal runs: the MMA warp consumed them).
      for (int s = 0; s < STAGES; ++s)
        if (armed_mask & (1u << s)) mbar_wait_drain(FULL_BAR(s), (armed_par >> s) & 1u, err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32(kBM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < total && ok; w += gridDim.x, ++it) {
        int m_tile, n_tile, split;
        decode_work(w, p, m_tile, n_tile, split);
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        const int acc = it & 1;
        const uint32_t acc_par = static_cast<uint32_t>((it >> 1) & 1);
        if (!mbar_wait(TEMPTY_BAR(acc), acc_par ^ 1u, err, kDevErrTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(FULL_BAR(stage), phase, err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            const uint64_t adesc = A_MN ? make_sw128_desc(sa + kk * 2048u, 8192u, 1024u)
                                        : make_sw128_desc(sa + kk * 32u, 16u, 1024u);
            const uint64_t bdesc = B_MN ? make_sw128_desc(sb + kk * 2048u, 8192u, 1024u)
                                        : make_sw128_desc(sb + kk * 32u, 16u, 1024u);
            tc_mma_f16(d_tmem, adesc, bdesc, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(EMPTY_BAR(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(TFULL_BAR(acc));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr int kParts = EPI_WARPS / 4;
    const int quad = warp & 3;
    const int part = (warp - kEpiWarp0) >> 2;
    int it = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x, ++it) {
      int m_tile, n_tile, split;
      decode_work(w, p, m_tile, n_tile, split);
      const int acc = it & 1;
      const uint32_t acc_par = static_cast<uint32_t>((it >> 1) & 1);
      if (!warp_wait(TFULL_BAR(acc), acc_par, err, kDevErrTimeoutTmemFull, lane)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      Epi::template run<BN, kParts>(ep, p, base_ptr + L::kEpiOffset, taddr, m_tile, n_tile, split,
                                    quad, part, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(TEMPTY_BAR(acc));
    }
    // Epilogues that store through TMA must see their bulk stores finish
    // reading shared memory before the CTA exits.
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (epi_cluster_exchange<Epi>::value) cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
#undef FULL_BAR
#undef EMPTY_BAR
#undef TFULL_BAR
#undef TEMPTY_BAR
}

// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2).  A cluster of two CTAs owns a
// 256 x BN output tile: CTA r loads A rows 128r..128r+127 of the pair tile and
// B columns (BN/2) r..(BN/2) r + BN/2 - 1 into its own shared memory (each
// load counted on the even CTA's stage barrier), one thread of the even CTA
// issues M = 256 MMAs that read both CTAs' stages, and each CTA's epilogue
// drains its own 128 accumulator rows from its own TMEM.  Per SM this halves
// the B traffic into shared memory for the same MMA rate.
// ---------------------------------------------------------------------------
template <int BN, int STAGES>
struct PairSmem {
  static constexpr int kABytes = kBM * kBK * 2;       // this CTA's 128 A rows
  static constexpr int kBBytes = (BN / 2) * kBK * 2;  // this CTA's half of B
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  static constexpr int kNumBars = 2 * STAGES + 4;
  static constexpr int kTmemSlotOffset = kBarOffset + kNumBars * 8;
  static constexpr int kEpiOffset = ((kTmemSlotOffset + 16 + 1023) / 1024) * 1024;
  // BN <= 256: two accumulators (epilogue overlaps the next tile); BN = 384:
  // one accumulator and two MMAs per K step (N = 256 + 128), for long-K GEMMs
  static constexpr int kAccs = BN <= 256 ? 2 : 1;
  static constexpr int kN0 = BN <= 256 ? BN : 256;  // first MMA of a K step
  static constexpr int kN1 = BN - kN0;              // second MMA (BN = 384)
  static constexpr int kTmemCols = kAccs * BN <= 256 ? 256 : 512;
  static_assert(BN == 128 || BN == 256 || BN == 384, "pair tile N");
};

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EPI_WARPS = 4>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(gemm_threads<EPI_WARPS>(), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA0,
                     const __grid_constant__ CUtensorMap tmA1,
                     const __grid_constant__ CUtensorMap tmA2,
                     const __grid_constant__ CUtensorMap tmB, const GemmParams p,
                     const __grid_constant__ typename Epi::Params ep) {
  using L = PairSmem<BN, STAGES>;
  static_assert(EPI_WARPS == 4 || EPI_WARPS == 8, "4 or 8 epilogue warps");
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t bar0 = base + L::kBarOffset;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + L::kTmemSlotOffset);
  int* err = p.err;
  // Dynamic shared memory starts at the same offset in both CTAs, so barrier
  // and stage offsets match across the pair.
#define FULL_BAR(s) (bar0 + 8u * (s))                    // even CTA: both halves landed
#define EMPTY_BAR(s) (bar0 + 8u * (STAGES + (s)))        // pair MMAs done with the stage
#define TFULL_BAR(a) (bar0 + 8u * (2 * STAGES + (a)))
#define TEMPTY_BAR(a) (bar0 + 8u * (2 * STAGES + 2 + (a)))  // even CTA: both epilogues

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(FULL_BAR(s), 1);
      mbar_init(EMPTY_BAR(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(TFULL_BAR(a), 1);
      mbar_init(TEMPTY_BAR(a), 2 * EPI_WARPS);
    }
    if constexpr (epi_has_init<Epi>::value) Epi::init(base_ptr + L::kEpiOffset);
    fence_mbar_init();
    prefetch_tensormap(&tmA0);
    if (p.a_seg1 > 0) {
      prefetch_tensormap(&tmA1);
      prefetch_tensormap(&tmA2);
    }
    prefetch_tensormap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), L::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // both CTAs' barriers initialised before any cross-CTA signal
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const int total = p.m_tiles * p.n_tiles * p.splits;  // m_tiles counts 256-row pair tiles
  const int w_first = static_cast<int>(cluster_id_x());
  const int w_step = static_cast<int>(num_clusters_x());

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_mask = 0, armed_par = 0;
      bool ok = true;
      for (int w = w_first; w < total && ok; w += w_step) {
        int m_pair, n_tile, split;
        decode_work(w, p, m_pair, n_tile, split);
        const int m0 = (2 * m_pair + static_cast<int>(rank)) * kBM;
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(EMPTY_BAR(stage), phase ^ 1u, err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) {
            mbar_arrive_expect_tx(FULL_BAR(stage), 2 * L::kStageBytes);
            armed_mask |= 1u << stage;
            armed_par = (armed_par & ~(1u << stage)) | (phase << stage);
          }
          const uint32_t full = mapa_shared(FULL_BAR(stage), 0);
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
          const int k0 = kb * kBK;
          if constexpr (!A_MN) {
            const CUtensorMap* mp = &tmA0;
            int kc = k0;
            if (p.a_seg1 > 0) select_segment(p, kc, mp, &tmA0, &tmA1, &tmA2);
            tma_load_2d_pair(sa, mp, kc, m0, full);
          } else {
#pragma unroll
            for (int i = 0; i < kBM / 64; ++i) {
              const CUtensorMap* mp = &tmA0;
              int mc = m0 + 64 * i;
              if (p.a_seg1 > 0) select_segment(p, mc, mp, &tmA0, &tmA1, &tmA2);
              tma_load_2d_pair(sa + i * 8192u, mp, mc, k0, full);
            }
          }
          // This CTA's half of B: columns (N0/2) r.. of the first MMA and, for
          // BN = 384, N0 + (N1/2) r.. of the second, as 64-column boxes
          // (K-major: 64-row boxes) stacked 8 KB apart.
          const int nb0 = (L::kN1 == 0 && p.b_pair_stride > 0)
                              ? n_tile * (BN / 2) + static_cast<int>(rank) * p.b_pair_stride
                              : n_tile * BN + static_cast<int>(rank) * (L::kN0 / 2);
#pragma unroll
          for (int i = 0; i < L::kN0 / 128; ++i) {
            if constexpr (!B_MN)
              tma_load_2d_pair(sb + i * 8192u, &tmB, k0, nb0 + 64 * i, full);
            else
              tma_load_2d_pair(sb + i * 8192u, &tmB, nb0 + 64 * i, k0, full);
          }
          if constexpr (L::kN1 > 0) {
            const int nb1 = n_tile * BN + L::kN0 + static_cast<int>(rank) * (L::kN1 / 2);
#pragma unroll
            for (int i = 0; i < L::kN1 / 128; ++i) {
              const uint32_t dst = sb + static_cast<uint32_t>(L::kN0 / 128 + i) * 8192u;
              if constexpr (!B_MN)
                tma_load_2d_pair(dst, &tmB, k0, nb1 + 64 * i, full);
              else
                tma_load_2d_pair(dst, &tmB, nb1 + 64 * i, k0, full);
            }
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Drain (even CTA): every armed stage, including the peer's half, has
      // landed before either CTA releases its shared memory.
      for (int s = 0; s < STAGES; ++s)
        if (armed_mask & (1u << s)) mbar_wait_drain(FULL_BAR(s), (armed_par >> s) & 1u, err);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ pair MMA issuer (even CTA)
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc0 = make_idesc_bf16_f32(2 * kBM, L::kN0, A_MN, B_MN);
      constexpr uint32_t idesc1 = make_idesc_bf16_f32(2 * kBM, L::kN1 > 0 ? L::kN1 : 16, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int w = w_first; w < total && ok; w += w_step, ++it) {
        int m_pair, n_tile, split;
        decode_work(w, p, m_pair, n_tile, split);
        const int kb0 = split * p.kb_per_split;
        const int kb1 = min(kb0 + p.kb_per_split, p.k_blocks);
        const int acc = L::kAccs == 2 ? (it & 1) : 0;
        const uint32_t acc_par = static_cast<uint32_t>(L::kAccs == 2 ? ((it >> 1) & 1) : (it & 1));
        if (!mbar_wait_cluster(TEMPTY_BAR(acc), acc_par ^ 1u, err, kDevErrTimeoutTmemEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_cluster(FULL_BAR(stage), phase, err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = base + stage * L::kStageBytes;
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            const uint64_t adesc = A_MN ? make_sw128_desc(sa + kk * 2048u, 8192u, 1024u)
                                        : make_sw128_desc(sa + kk * 32u, 16u, 1024u);
            const uint64_t bdesc = B_MN ? make_sw128_desc(sb + kk * 2048u, 8192u, 1024u)
                                        : make_sw128_desc(sb + kk * 32u, 16u, 1024u);
            const uint32_t accum = (kb > kb0 || kk > 0) ? 1u : 0u;
            tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc0, accum);
            if constexpr (L::kN1 > 0) {
              // second MMA: columns [256, BN); its B half starts after the first's
              constexpr uint32_t off = static_cast<uint32_t>(L::kN0 / 2) * 128u;
              const uint64_t bdesc1 = B_MN ? make_sw128_desc(sb + off + kk * 2048u, 8192u, 1024u)
                                           : make_sw128_desc(sb + off + kk * 32u, 16u, 1024u);
              tc_mma_f16_pair(d_tmem + static_cast<uint32_t>(L::kN0), adesc, bdesc1, idesc1, accum);
            }
          }
          tc_commit_pair(EMPTY_BAR(stage));
          tc_commit_pair(mapa_shared(EMPTY_BAR(stage), 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit_pair(TFULL_BAR(acc));
        tc_commit_pair(mapa_shared(TFULL_BAR(acc), 1));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    constexpr int kParts = EPI_WARPS / 4;
    const int quad = warp & 3;
    const int part = (warp - kEpiWarp0) >> 2;
    int it = 0;
    for (int w = w_first; w < total; w += w_step, ++it) {
      int m_pair, n_tile, split;
      decode_work(w, p, m_pair, n_tile, split);
      const int acc = L::kAccs == 2 ? (it & 1) : 0;
      const uint32_t acc_par = static_cast<uint32_t>(L::kAccs == 2 ? ((it >> 1) & 1) : (it & 1));
      if (!warp_wait(TFULL_BAR(acc), acc_par, err, kDevErrTimeoutTmemFull, lane)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      Epi::template run<BN, kParts>(ep, p, base_ptr + L::kEpiOffset, taddr,
                                    2 * m_pair + static_cast<int>(rank), n_tile, split, quad, part,
                                    lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(TEMPTY_BAR(acc), 0));
    }
    if (lane == 0) bulk_wait_group_all();
    __syncwarp();
  }

  // Neither CTA may leave while the other can still signal its barriers or the
  // pair MMAs can still read its shared memory.
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

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

// Encode a 2-D bf16 tensor map with 128-byte swizzle.
//   inner: elements along the contiguous dimension, outer: number of rows,
//   ld: row stride in elements, box = {64, box_outer}.
bool encode_bf16_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                     uint64_t ld, uint32_t box_outer);

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EPI_WARPS = 4>
int launch_gemm_sm100(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& a2,
                      const CUtensorMap& b, const GemmParams& p, const typename Epi::Params& ep,
                      cudaStream_t stream, int kernel_id) {
  using L = GemmSmem<BN, STAGES>;
  auto kern = gemm_sm100_kernel<BN, STAGES, A_MN, B_MN, Epi, EPI_WARPS>;
  const int smem = L::kEpiOffset + Epi::template smem_bytes<EPI_WARPS>() + 1024;
  static_assert(L::kEpiOffset + Epi::template smem_bytes<EPI_WARPS>() + 1024 <= 232448,
                "shared memory budget exceeded");
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  const int total = p.m_tiles * p.n_tiles * p.splits;
  if (total <= 0) return HLM_OK;
  int grid = num_sms_of_current_device();
  if (grid > total) grid = total;
  {
    LaunchScope scope(kernel_id, stream);
    kern<<<grid, gemm_threads<EPI_WARPS>(), smem, stream>>>(a0, a1, a2, b, p, ep);
  }
  return launch_status();
}

// Cluster launch of the single-CTA kernel: clusters of `cluster` CTAs (grid a
// multiple of it), for
// epilogues that exchange data across the cluster.  With p.n_tiles == cluster
// and p.splits == 1, the CTAs of a cluster take the n tiles of one m tile
// together (work index w = m_tile * n_tiles + n_tile, stepped by the grid).
template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EPI_WARPS = 4>
int launch_gemm_cluster(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& a2,
                        const CUtensorMap& b, const GemmParams& p, const typename Epi::Params& ep,
                        int cluster, cudaStream_t stream, int kernel_id) {
  using L = GemmSmem<BN, STAGES>;
  auto kern = gemm_sm100_kernel<BN, STAGES, A_MN, B_MN, Epi, EPI_WARPS>;
  const int smem = L::kEpiOffset + Epi::template smem_bytes<EPI_WARPS>() + 1024;
  static_assert(L::kEpiOffset + Epi::template smem_bytes<EPI_WARPS>() + 1024 <= 232448,
                "shared memory budget exceeded");
  if (cluster < 1 || cluster > 8 || p.n_tiles != cluster || p.splits != 1) return HLM_ERR_INVALID_ARG;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  if (p.m_tiles <= 0) return HLM_OK;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(gemm_threads<EPI_WARPS>(), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // As many clusters as fit on the GPU at once (cluster placement within GPCs can
  // leave SMs unused, e.g. 45 clusters of three CTAs on 148 SMs): a persistent
  // cluster beyond that would start only when another has finished all its tiles.
  int clusters = num_sms_of_current_device() / cluster;
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * cluster), 1, 1);
  int fit = 0;
  if (cudaOccupancyMaxActiveClusters(&fit, kern, &cfg) == cudaSuccess && fit > 0 && fit < clusters)
    clusters = fit;
  if (clusters > p.m_tiles) clusters = p.m_tiles;
  if (clusters < 1) clusters = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * cluster), 1, 1);
  {
    LaunchScope scope(kernel_id, stream);
    if (cudaLaunchKernelEx(&cfg, kern, a0, a1, a2, b, p, ep) != cudaSuccess) return HLM_ERR_LAUNCH;
  }
  return launch_status();
}

// Pair launch: one cluster of two CTAs per two SMs, persistent over the
// 256 x BN pair tiles (p.m_tiles counts pair tiles: gemm_tiling_pair).
template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi, int EPI_WARPS = 4>
int launch_gemm_pair(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& a2,
                     const CUtensorMap& b, const GemmParams& p, const typename Epi::Params& ep,
                     cudaStream_t stream, int kernel_id) {
  using L = PairSmem<BN, STAGES>;
  auto kern = gemm_pair_kernel<BN, STAGES, A_MN, B_MN, Epi, EPI_WARPS>;
  const int smem = L::kEpiOffset + Epi::template smem_bytes<EPI_WARPS>() + 1024;
  static_assert(L::kEpiOffset + Epi::template smem_bytes<EPI_WARPS>() + 1024 <= 232448,
                "shared memory budget exceeded");
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  const int total = p.m_tiles * p.n_tiles * p.splits;
  if (total <= 0) return HLM_OK;
  int pairs = num_sms_of_current_device() / 2;
  if (pairs > total) pairs = total;
  if (pairs < 1) pairs = 1;
  {
    LaunchScope scope(kernel_id, stream);
    kern<<<2 * pairs, gemm_threads<EPI_WARPS>(), smem, stream>>>(a0, a1, a2, b, p, ep);
  }
  return launch_status();
}

// Fill the tiling fields of GemmParams.
inline void gemm_tiling(GemmParams& p, int M, int N, int K, int BN, int splits) {
  p.M = M;
  p.N = N;
  p.K = K;
  p.m_tiles = (M + kBM - 1) / kBM;
  p.n_tiles = (N + BN - 1) / BN;
  p.k_blocks = (K + kBK - 1) / kBK;
  if (splits < 1) splits = 1;
  if (splits > p.k_blocks) splits = p.k_blocks;
  p.kb_per_split = (p.k_blocks + splits - 1) / splits;
  p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  p.a_seg1 = 0;
  p.a_seg2 = 0;
  p.b_pair_stride = 0;
}

// Same for the pair kernel: m_tiles counts 256-row pair tiles.
inline void gemm_tiling_pair(GemmParams& p, int M, int N, int K, int BN, int splits) {
  gemm_tiling(p, M, N, K, BN, splits);
  p.m_tiles = (M + 2 * kBM - 1) / (2 * kBM);
}

// ---------------------------------------------------------------------------
// Epilogue: store D (bf16 or fp32), optional accumulate, optional split-K slab
// ---------------------------------------------------------------------------
struct EpiStore {
  struct Params {
    void* d;
    int64_t ldd;
    int64_t split_stride;  // elements between split-K slabs (fp32 partials)
    int dtype;             // HLM_BF16 or HLM_F32
    int accumulate;        // 1: D += acc (read-modify-write); 2 (fp32 only): D += acc by
                           // atomic reductions in L2, for split-K partials of one D
    int vec_ok;            // ldd % 8 == 0 and d 16-byte aligned
    const float* alpha;    // optional device scalar: D = alpha * acc (+ D)
  };
  template <int EPI_WARPS>
  static constexpr int smem_bytes() {
    return 0;
  }

  // Warp `part` of kParts sharing this lane quadrant takes every kParts-th
  // 32-column group.
  template <int BN, int kParts>
  static HLM_DEVICE void run(const Params& ep, const GemmParams& p, uint8_t* /*smem*/,
                             uint32_t taddr, int m_tile, int n_tile, int split, int quad, int part,
                             int lane) {
    const int row = m_tile * kBM + quad * 32 + lane;
    const bool row_ok = row < p.M;
    const float alpha = ep.alpha != nullptr ? *ep.alpha : 1.0f;
#pragma unroll 1
    for (int c = part; c < BN / 32; c += kParts) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c * 32), r);
      tmem_ld_wait();
      const int col0 = n_tile * BN + c * 32;
      if (!row_ok || col0 >= p.N) continue;
      if (ep.alpha != nullptr) {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha);
      }
      const bool full = ep.vec_ok && (col0 + 32 <= p.N);
      if (ep.dtype == HLM_F32) {
        float* d = static_cast<float*>(ep.d) + static_cast<int64_t>(split) * ep.split_stride +
                   static_cast<int64_t>(row) * ep.ldd + col0;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                   __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
            if (ep.accumulate == 2) {
              asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(d + j), "f"(v.x), "f"(v.y),
                           "f"(v.z), "f"(v.w)
                           : "memory");
              continue;
            }
            if (ep.accumulate) {
              const float4 o = *reinterpret_cast<const float4*>(d + j);
              v.x += o.x;
              v.y += o.y;
              v.z += o.z;
              v.w += o.w;
            }
            *reinterpret_cast<float4*>(d + j) = v;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (col0 + j < p.N) {
              float v = __uint_as_float(r[j]);
              if (ep.accumulate == 2) {
                atomicAdd(d + j, v);
                continue;
              }
              if (ep.accumulate) v += d[j];
              d[j] = v;
            }
          }
        }
      } else {
        __nv_bfloat16* d = static_cast<__nv_bfloat16*>(ep.d) + static_cast<int64_t>(row) * ep.ldd + col0;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(r[j + i]);
            if (ep.accumulate) {
              Vec16<__nv_bfloat16> o;
              o.raw = *reinterpret_cast<const uint4*>(d + j);
              float of[8];
              o.to_float(of);
#pragma unroll
              for (int i = 0; i < 8; ++i) f[i] += of[i];
            }
            Vec16<__nv_bfloat16> v;
            v.from_float(f);
            *reinterpret_cast<uint4*>(d + j) = v.raw;
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (col0 + j < p.N) {
              float v = __uint_as_float(r[j]);
              if (ep.accumulate) v += __bfloat162float(d[j]);
              d[j] = __float2bfloat16_rn(v);
            }
          }
        }
      }
    }
  }
};

}  // namespace hlm
