// Causal (optionally sliding-window) attention forward on tcgen05: the
// attention core the reference reaches through kernels.scaled_dot_product_attention
// (kernels.py:774-847; FlashAttention window (w - 1, 0), kernels.py:839; the
// per-layer windows of config.py:184-191), for head_dim 128 and bf16.
//
//   out[b, t, h, :] = softmax_k( q[b,t,h,:] . k[b,k,hk,:] * scale, 0 <= t - k < w ) @ v[b,k,hk,:]
//   lse[b, h, t]    = log(sum_k exp(q . k * scale))          (natural log, fp32)
//
// q, k, v, out are [B, T, H(k), 128] bf16 (the layout the QKV kernel writes), so
// no transposes are needed; grouped-query heads map h -> h / (H / Hk).
//
// One CTA takes two query tiles of 128 rows of one (b, h) (K and V are read once
// for both) and walks the key tiles of 128 from the first the window reaches to
// the last diagonal:
//   warp 0  TMA producer: Q of both tiles, then K_t / V_t through a five-slot ring
//   warp 1  TMEM owner and MMA issuer: S_w = Q_w K_t^T (M=N=K=128) into tile w's
//           score columns; O_w += P_w V_t with P_w read from tensor memory; per key
//           tile PV_0, S_0(next), PV_1, S_1(next), so that one group's softmax
//           runs while the tensor cores do the other group's two MMAs
//   warps 4-7, 8-11  softmax of tile 0 / 1, one query row per thread: the score row
//           into registers, exp2 of the scaled, masked scores against a running
//           reference max m (no row max once every row has one; the exact path,
//           with the row max and m moved only when exceeded by more than 8, takes a
//           row's first key tile and any half whose sum leaves [0, 2^64]), running
//           sum, P as bf16 pairs over the first 64 score columns published per key
//           half, and, when m moves, the output row rescaled in TMEM (tcgen05.ld /
//           st); at the end out = O / l through TMA stores and lse = (m + log2 l) ln 2.
// S_w of the next key tile overwrites P_w, so it is issued after PV_w; MMAs of one
// thread run in order, so the commit that publishes S_w also covers PV_w (its O
// may be rescaled and its P overwritten).  Every wait is bounded.
#include "gemm_sm100.cuh"

namespace hlm {

HLM_DEVICE void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
HLM_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Waits poll the barrier with mbarrier.test_wait, back to back: every wait of the
// MMA issuer is on the critical chain, and a __nanosleep between polls (even of
// 32 ns) measured about 1000 cycles late.  Suspending in mbarrier.try_wait
// measured the same as polling.  Every wait is bounded.
HLM_DEVICE bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
HLM_DEVICE bool mbar_poll(uint32_t bar, uint32_t parity, int* err, int code) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > kWaitTimeoutNs) {
      record_error(err, code);
      return false;
    }
  }
}
HLM_DEVICE bool warp_poll(uint32_t bar, uint32_t parity, int* err, int code, int lane) {
  int ok = 1;
  if (lane == 0) ok = mbar_poll(bar, parity, err, code) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// D[tmem] (+)= A[tmem] * B[smem]: the A operand (M = 128 rows, K = 16 bf16 per
// instruction) read from tensor memory, two elements per 32-bit column.
HLM_DEVICE void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic, one instruction for two lanes of
// work; each element rounds exactly as the scalar instruction) and the
// three-input max: the softmax is bound by its instruction issue, not by the
// exp2 unit.
HLM_DEVICE uint64_t f32x2_splat(float v) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(v));
  return r;
}
// (d0, d1) = (a0, a1) * b2 + c2
HLM_DEVICE void fma_f32x2(float& d0, float& d1, float a0, float a1, uint64_t b2, uint64_t c2) {
  asm("{\n\t.reg .b64 ra, rd;\n\tmov.b64 ra, {%2, %3};\n\t"
      "fma.rn.f32x2 rd, ra, %4, %5;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "l"(b2), "l"(c2));
}
// (s0, s1) += (a0, a1)
HLM_DEVICE void add_f32x2(float& s0, float& s1, float a0, float a1) {
  asm("{\n\t.reg .b64 rs, ra;\n\tmov.b64 rs, {%0, %1};\n\tmov.b64 ra, {%2, %3};\n\t"
      "add.rn.f32x2 rs, rs, ra;\n\tmov.b64 {%0, %1}, rs;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "f"(a0), "f"(a1));
}
HLM_DEVICE float max3_f32(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// Keys of one 32-key chunk outside the causal window [qpos - window + 1, qpos]
// set to -inf (tiles the mask reaches only).
HLM_DEVICE void att_chunk_mask(uint32_t (&xc)[32], int key0c, int qpos, int window) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int k = key0c + i;
    if (!(k <= qpos && qpos - k < window)) xc[i] = __float_as_uint(-INFINITY);
  }
}
// Max of the raw scores of one 32-key chunk into eight partial maxima (the
// reduction would otherwise be one dependent chain).
HLM_DEVICE void att_chunk_max(const uint32_t (&xc)[32], float (&mxp)[8]) {
#pragma unroll
  for (int i = 0; i < 32; i += 2)
    mxp[(i >> 1) & 7] = max3_f32(mxp[(i >> 1) & 7], __uint_as_float(xc[i]), __uint_as_float(xc[i + 1]));
}
HLM_DEVICE float att_max_of(const float (&mxp)[8]) {
  return fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])), fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
}
// Max of the raw scores over `n` 32-key chunks starting at x[c0].
template <int C0, int N>
HLM_DEVICE float att_chunks_max(const uint32_t (&x)[4][32]) {
  float mxp[8];
#pragma unroll
  for (int u8 = 0; u8 < 8; ++u8) mxp[u8] = -INFINITY;
#pragma unroll
  for (int c = C0; c < C0 + N; ++c) att_chunk_max(x[c], mxp);
  return att_max_of(mxp);
}
// p = 2^(x * sc + nm) over one 32-key chunk: bf16 pairs for the PV MMA into
// pk[0..15] and the fp32 sums into r0 / r1 (the log-sum-exp the backward
// recomputes P from takes the fp32 values).
HLM_DEVICE void att_exp_chunk(const uint32_t (&xc)[32], uint64_t sc2, uint64_t nm2, uint32_t* pk, float (&r0)[4],
                              float (&r1)[4]) {
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    float a0, a1;
    fma_f32x2(a0, a1, __uint_as_float(xc[i]), __uint_as_float(xc[i + 1]), sc2, nm2);
    const float e0 = ex2_ftz(a0);
    const float e1 = ex2_ftz(a1);
    add_f32x2(r0[(i >> 1) & 3], r1[(i >> 1) & 3], e0, e1);
    pk[i / 2] = pack_bf16x2(e0, e1);
  }
}
// Two chunks (one key half): P pairs into pk[0..31], returns the fp32 sum.
HLM_DEVICE float att_exp_half(const uint32_t (&xa)[32], const uint32_t (&xb)[32], uint64_t sc2, uint64_t nm2,
                              uint32_t (&pk)[32]) {
  float r0[4], r1[4];
#pragma unroll
  for (int u4 = 0; u4 < 4; ++u4) r0[u4] = r1[u4] = 0.0f;
  att_exp_chunk(xa, sc2, nm2, pk, r0, r1);
  att_exp_chunk(xb, sc2, nm2, pk + 16, r0, r1);
  return ((r0[0] + r1[0]) + (r0[1] + r1[1])) + ((r0[2] + r1[2]) + (r0[3] + r1[3]));
}
// One thread's output row in tensor memory scaled by alpha.
HLM_DEVICE void att_rescale_o(uint32_t taddr, float alpha) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t o[32];
    tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(c * 32), o);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
    tmem_st_32x32b_x32(taddr + static_cast<uint32_t>(c * 32), o);
  }
}

constexpr int kAttD = 128;           // head dim
constexpr int kAttBQ = 128;          // query rows per tile (two tiles per CTA)
constexpr int kAttBK = 128;          // keys per tile
constexpr int kAttAtom = 128 * 128;  // one 128-row x 64-column bf16 swizzle atom (16 KB)
constexpr int kAttTile = 2 * kAttAtom;  // one 128 x 128 bf16 tile (32 KB)
constexpr int kAttThreads = 384;
// Register split: launched at kAttLaunchRegs per thread (384 x 168 = 64512, the
// whole budget of one CTA per SM); the first warpgroup (TMA producer, MMA issuer,
// two idle warps) gives registers back so that the two softmax warpgroups hold a
// 128-entry score row and its packed P without spilling.  The shares add up to
// the launch's total: 128 x 56 + 256 x 224 = 64512.  The host refuses to launch if
// the compiled kernel's register count differs (a larger share would then wait
// forever).
constexpr int kAttLaunchRegs = 168;
constexpr int kAttIssuerRegs = 56;
constexpr int kAttSoftmaxRegs = 224;
static_assert(128 * kAttIssuerRegs + 256 * kAttSoftmaxRegs <= kAttThreads * kAttLaunchRegs, "register split");
struct AttSmem {
  static constexpr int kQ = 0;                   // Q of the two query tiles (K-major atoms d 0-63, 64-127)
  // one ring of tile slots for K_0, V_0, K_1, V_1, ... (item n = 2t for K_t,
  // 2t + 1 for V_t, in slot n % kSlots): K as two K-major atoms, V as MN-major
  // 64 x 64 blocks
  static constexpr int kSlots = 5;
  static constexpr int kKV = kQ + 2 * kAttTile;
  static constexpr int kBars = kKV + kSlots * kAttTile;
  // q_full, kv_full[5], kv_empty[5], s_full[2], p_lo[2], p_hi[2], o_done[2], pvlo_done[2]
  static constexpr int kNumBars = 1 + 2 * kSlots + 10;
  static constexpr int kTmemSlot = kBars + kNumBars * 8;
  static constexpr int kBytes = kTmemSlot + 16;
};

struct AttParams {
  int B, T, H, Hk;
  int window;       // keys with t - k < window (window >= T: full causal)
  int q_tiles;      // T / 128
  int q_pairs;      // ceil(q_tiles / 2): work items per (b, h)
  float scale_log2; // softmax scale * log2(e)
  float* lse;       // [B, H, T]
  int* err;
};

__global__ void __launch_bounds__(kAttThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmVk, const __grid_constant__ CUtensorMap tmO,
                    const AttParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = p.err;

  // work item: query tiles 2i and 2i + 1 of one (b, h).  Items are ordered by
  // pair index over the whole grid, highest (longest under the causal mask)
  // first, so that CTAs start longest-first and the last wave holds short items.
  const int item = static_cast<int>(blockIdx.x);
  const int n_bh = p.B * p.H;
  const int pair = p.q_pairs - 1 - item / n_bh;
  const int bh = item - (item / n_bh) * n_bh;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int hk = h / (p.H / p.Hk);
  const int qt0 = 2 * pair;
  const bool has1 = qt0 + 1 < p.q_tiles;
  auto first_tile = [&](int q) { return max(0, q * kAttBQ - p.window + 1) / kAttBK; };
  const int j_first = first_tile(qt0);                 // key tiles j_first .. j_last, t = j - j_first
  const int j_last = has1 ? qt0 + 1 : qt0;
  const int nkv = j_last - j_first + 1;
  // query tile w covers key tiles t0(w) .. t1(w)
  const int t_lo1 = first_tile(qt0 + 1) - j_first;
  auto t0 = [&](int w) { return w == 0 ? 0 : t_lo1; };
  auto t1 = [&](int w) { return qt0 + w - j_first; };
  auto covers = [&](int w, int t) { return (w == 0 || has1) && t >= t0(w) && t <= t1(w); };

  const uint32_t bar0 = base + AttSmem::kBars;
  const uint32_t q_full = bar0;
  // ring item n: its slot, its landing barrier and the barrier that frees it
  constexpr int kS = AttSmem::kSlots;
  auto slot_addr = [&](int n) { return base + AttSmem::kKV + static_cast<uint32_t>((n % kS) * kAttTile); };
  auto kv_full = [&](int n) { return bar0 + 8u * static_cast<uint32_t>(1 + n % kS); };
  auto kv_empty = [&](int n) { return bar0 + 8u * static_cast<uint32_t>(1 + kS + n % kS); };
  auto kv_par = [&](int n) { return static_cast<uint32_t>((n / kS) & 1); };  // phase of item n's use
  constexpr int kB = 1 + 2 * kS;
  auto s_full = [&](int w) { return bar0 + 8u * (kB + w); };
  // P of keys 0-63 / 64-127 of tile w's current key tile written
  auto p_lo = [&](int w) { return bar0 + 8u * (kB + 2 + w); };
  auto p_hi = [&](int w) { return bar0 + 8u * (kB + 4 + w); };
  auto o_done = [&](int w) { return bar0 + 8u * (kB + 6 + w); };
  // PV of the first key half of tile w's current key tile completed
  auto pvlo_done = [&](int w) { return bar0 + 8u * (kB + 8 + w); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + AttSmem::kTmemSlot);

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int n = 0; n < kS; ++n) {
      mbar_init(kv_full(n), 1);
      mbar_init(kv_empty(n), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(s_full(s), 1);
      mbar_init(p_lo(s), 4);  // the four warps of that tile's softmax group
      mbar_init(p_hi(s), 4);
      mbar_init(o_done(s), 1);
      mbar_init(pvlo_done(s), 1);
    }
    fence_mbar_init();
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmVk);
    prefetch_tensormap(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // TMEM columns: S of tile 0 / 1 (P overwrites its first 64 columns as bf16
  // pairs), then O of tile 0 / 1
  auto t_s = [&](int w) { return tmem_base + 128u * static_cast<uint32_t>(w); };
  auto t_o = [&](int w) { return tmem_base + 256u + 128u * static_cast<uint32_t>(w); };
  const int row_k0 = b * p.T;  // first key row of this sequence in the [B*T, H*D] view

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kAttIssuerRegs));
  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      const int nq = has1 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, static_cast<uint32_t>(nq * kAttTile));
      for (int w = 0; w < nq; ++w) {
        const int row_q = row_k0 + (qt0 + w) * kAttBQ;
        const uint32_t dst = base + AttSmem::kQ + static_cast<uint32_t>(w * kAttTile);
        tma_load_2d(dst, &tmQ, h * kAttD, row_q, q_full);
        tma_load_2d(dst + kAttAtom, &tmQ, h * kAttD + 64, row_q, q_full);
      }
      // K_t and V_t into the ring, running up to kSlots items ahead of the MMAs
      int issued = 0;  // ring items whose loads were issued
      for (int n = 0; n < 2 * nkv && ok; ++n) {
        if (n >= kS && !mbar_poll(kv_empty(n), kv_par(n) ^ 1u, err, kDevErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        const int key0 = row_k0 + (j_first + (n >> 1)) * kAttBK;
        const uint32_t dst = slot_addr(n);
        mbar_arrive_expect_tx(kv_full(n), kAttTile);
        if ((n & 1) == 0) {
          tma_load_2d(dst, &tmK, hk * kAttD, key0, kv_full(n));
          tma_load_2d(dst + kAttAtom, &tmK, hk * kAttD + 64, key0, kv_full(n));
        } else {
          // V: MN-major blocks [64 keys][64 d]: key block kb at 16 KB, d block i at 8 KB
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int i = 0; i < 2; ++i)
              tma_load_2d(dst + static_cast<uint32_t>(kb * 16384 + i * 8192), &tmVk, hk * kAttD + 64 * i,
                          key0 + 64 * kb, kv_full(n));
        }
        issued = n + 1;
      }
      // every load issued has landed before the CTA can exit (after an error too)
      mbar_wait_drain(q_full, 0u, err);
      for (int n = max(0, issued - kS); n < issued; ++n) mbar_wait_drain(kv_full(n), kv_par(n), err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, 128, false, true);
      bool ok = mbar_poll(q_full, 0u, err, kDevErrTimeoutFull);
      // The K and V tiles an MMA pair needs are waited for before the P it waits
      // on (they have almost always landed by then), so that nothing but the
      // softmax's arrival stands between one group's P and its two MMAs.
      int k_ready = -1, v_ready = -1;  // highest key tile whose K / V has been seen landed
      auto wait_k = [&](int t) -> bool {
        if (t <= k_ready) return true;
        k_ready = t;
        return mbar_poll(kv_full(2 * t), kv_par(2 * t), err, kDevErrTimeoutFull);
      };
      auto wait_v = [&](int t) -> bool {
        if (t <= v_ready) return true;
        v_ready = t;
        return mbar_poll(kv_full(2 * t + 1), kv_par(2 * t + 1), err, kDevErrTimeoutFull);
      };
      // S_w = Q_w K_t^T into tile w's score columns (K_t has landed)
      auto issue_s = [&](int w, int t) {
        const uint32_t qa = base + AttSmem::kQ + static_cast<uint32_t>(w * kAttTile);
        const uint32_t kb = slot_addr(2 * t);
#pragma unroll
        for (int kk = 0; kk < kAttD / kUmmaK; ++kk) {
          const uint32_t atom = static_cast<uint32_t>((kk >> 2) * kAttAtom + (kk & 3) * 32);
          tc_mma_f16(t_s(w), make_sw128_desc(qa + atom, 16u, 1024u), make_sw128_desc(kb + atom, 16u, 1024u),
                     idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full(w));
      };
      // O_w += P_w V_t over keys 64 * half .. + 63, P_w read from tensor memory
      // (that half of P_w and V_t ready)
      auto issue_pv = [&](int w, int t, int half) {
        const int u = t - t0(w);
        const uint32_t vb = slot_addr(2 * t + 1);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = 4 * half + k4;
          tc_mma_f16_ts(t_o(w), t_s(w) + static_cast<uint32_t>(kk * 8),
                        make_sw128_desc(vb + static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 2048), 8192u, 1024u),
                        idesc_o, (u > 0 || kk > 0) ? 1u : 0u);
        }
        if (half == 1 && t == t1(w)) tc_commit(o_done(w));
      };
      for (int w = 0; w < 2 && ok; ++w)
        if (covers(w, 0)) {
          if (!(ok = wait_k(0))) break;
          tc_fence_after();
          issue_s(w, 0);
        }
      if (ok) tc_commit(kv_empty(0));
      // per key tile: PV_0, S_0 of the next tile, PV_1, S_1 of the next tile, so
      // that one group's softmax overlaps the other's two MMAs
      for (int t = 0; t < nkv && ok; ++t) {
        for (int w = 0; w < 2 && ok; ++w) {
          const bool pv = covers(w, t), next = covers(w, t + 1);
          if (pv && !(ok = wait_v(t))) break;
          if (next && !(ok = wait_k(t + 1))) break;
          if (!pv && !next) continue;
          if (pv) {
            // the first half of P is ready while the softmax still computes the second
            const uint32_t par = static_cast<uint32_t>((t - t0(w)) & 1);
            if (!(ok = mbar_poll(p_lo(w), par, err, kDevErrTimeoutFull))) break;
            tc_fence_after();
            issue_pv(w, t, 0);
            tc_commit(pvlo_done(w));
            if (!(ok = mbar_poll(p_hi(w), par, err, kDevErrTimeoutFull))) break;
            tc_fence_after();
            issue_pv(w, t, 1);
          } else {
            tc_fence_after();
          }
          if (next) issue_s(w, t + 1);
        }
        if (!ok) break;
        // K_{t+1} is free once both groups' S MMAs on it complete, V_t once both PVs do
        if (t + 1 < nkv) tc_commit(kv_empty(2 * t + 2));
        tc_commit(kv_empty(2 * t + 1));
      }
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kAttSoftmaxRegs));
    // ------------------------------------------------------------ softmax groups
    const int w = (warp - 4) >> 2;   // query tile of this group
    const int quad = warp & 3;       // TMEM lane quarter this warp may access
    const int r = quad * 32 + lane;  // row of the tile
    const int q0 = (qt0 + w) * kAttBQ;
    const int qpos = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float sc = p.scale_log2;
    float m = -INFINITY, l = 0.0f;  // reference max (log2 domain) and row sum
    bool ok = w == 0 || has1;
    const int nu = ok ? t1(w) - t0(w) + 1 : 0;
    for (int u = 0; u < nu; ++u) {
      const int key0 = (j_first + t0(w) + u) * kAttBK;
      if (!warp_poll(s_full(w), static_cast<uint32_t>(u & 1), err, kDevErrTimeoutTmemFull, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const bool full_tile = key0 + kAttBK - 1 <= q0 && q0 + kAttBQ - 1 - key0 < p.window;
      uint32_t x[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_s(w) + lane_off + static_cast<uint32_t>(c * 32), x[c]);
      tmem_ld_wait();
      if (!full_tile) {
#pragma unroll
        for (int c = 0; c < 4; ++c) att_chunk_mask(x[c], key0 + 32 * c, qpos, p.window);
      }
      const uint64_t sc2 = f32x2_splat(sc);
      // P over the first 64 score columns (S has been read; PV of the previous
      // tile, which read the previous P there, completed before this S did),
      // published per key half so that the PV MMA of the first half overlaps the
      // exp2 of the second.
      //
      // Fast path, once every row of the warp has a finite reference m: the
      // exponents s * scale - m take m as it stands, with no row max (the max is
      // a large share of the softmax's instructions).  Softmax does not depend on
      // the reference; it only has to keep the terms in range, so a half whose sum
      // exceeds 2^64 (or is inf / NaN) in any row of the warp goes the exact way.
      // Exact path (each row's first key tile, or a first half out of range): the
      // row max moves the reference when it exceeds it by more than 8, and O and l
      // are rescaled (alpha) on those moves; alpha is 0 when the row had no valid
      // key before (its O row and l are 0).
      float alpha = 1.0f, rs0 = 0.0f;
      uint32_t pk[32];
      bool exact = u == 0 || __any_sync(0xffffffffu, m == -INFINITY);
      if (!exact) {
        rs0 = att_exp_half(x[0], x[1], sc2, f32x2_splat(-m), pk);
        exact = __any_sync(0xffffffffu, !(rs0 <= 0x1p64f));
      }
      if (exact) {
        const float mx = sc * att_chunks_max<0, 4>(x);
        if (mx > m + 8.0f) {
          alpha = ex2_ftz(m - mx);
          m = mx;
        }
        // O is overwritten at u == 0; PV of the previous tile has completed
        if (u > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) att_rescale_o(t_o(w) + lane_off, alpha);
        rs0 = att_exp_half(x[0], x[1], sc2, f32x2_splat(m == -INFINITY ? 0.0f : -m), pk);
      }
      tmem_st_32x32b_x32(t_s(w) + lane_off, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_lo(w));
      float rs1 = att_exp_half(x[2], x[3], sc2, f32x2_splat(m == -INFINITY ? 0.0f : -m), pk);
      if (__any_sync(0xffffffffu, !(rs1 <= 0x1p64f))) {
        // A term of the second half left the range after the first half was
        // published (only on the fast path: the exact path keeps terms <= 2^8).
        // Move the reference to the second half's max (the first half's terms, in
        // range under the old reference, only shrink), wait for the first half's
        // PV, rescale O and the first half's sum, and recompute the second half.
        const float mx = fmaxf(m, sc * att_chunks_max<2, 2>(x));
        const float a2 = ex2_ftz(m - mx);
        m = mx;
        if (!warp_poll(pvlo_done(w), static_cast<uint32_t>(u & 1), err, kDevErrTimeoutTmemFull, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
        att_rescale_o(t_o(w) + lane_off, a2);
        alpha *= a2;
        rs0 *= a2;
        rs1 = att_exp_half(x[2], x[3], sc2, f32x2_splat(-m), pk);
      }
      tmem_st_32x32b_x32(t_s(w) + lane_off + 32u, pk);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_hi(w));
      l = alpha * l + (rs0 + rs1);
    }
    if (ok && warp_poll(o_done(w), 0u, err, kDevErrTimeoutTmemFull, lane)) {
      tc_fence_after();
      const float inv_l = 1.0f / l;
      // out row -> this tile's Q buffer (free: its last S MMA completed before the
      // last PV did), as two 32 x 64 boxes per warp per 64-column half, then TMA stores
      const uint32_t stage =
          base + AttSmem::kQ + static_cast<uint32_t>(w * kAttTile + quad * 2 * 32 * 128);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o(w) + lane_off + static_cast<uint32_t>(c * 32), o);
        tmem_ld_wait();
        const uint32_t box = stage + static_cast<uint32_t>((c >> 1) * 32 * 128);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (c & 1) * 4 + q;
          const uint4 v4 = make_uint4(pack_bf16x2(__uint_as_float(o[8 * q]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l),
                                      pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l),
                                      pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l),
                                      pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l));
          st_shared_v4(box + static_cast<uint32_t>(lane * 128 + ((ch ^ (lane & 7)) << 4)), v4);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      const int row_q = row_k0 + q0;
      if (lane == 0) {
        tma_store_2d(&tmO, h * kAttD, row_q + quad * 32, stage);
        tma_store_2d(&tmO, h * kAttD + 64, row_q + quad * 32, stage + 32 * 128);
        bulk_commit_group();
      }
      p.lse[(static_cast<int64_t>(b) * p.H + h) * p.T + qpos] = (m + __log2f(l)) * 0.6931471805599453f;
      if (lane == 0) bulk_wait_group_all();
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}


// ---------------------------------------------------------------------------
// Attention backward (the same masks, head_dim 128, H == Hk):
//   D[b,h,t]  = sum_d dO . O,  L[b,h,t] = lse log2 e           (attn_bwd_prep_kernel)
//   P^T       = 2^(S^T scale log2 e - L), S^T = K Q^T, masked
//   dP^T      = V dO^T,   dS^T = P^T (dP^T - D)
//   dV += P^T dO,   dK += scale dS^T Q,   dQ^T += scale K^T dS^T  (attn_bwd_kernel)
// One CTA per (b, h, key tile j of 128 keys) walks the 64-query blocks the window
// reaches from tile j.  Tensor memory: two stages of [S^T | dP^T] (64 + 64
// columns each), dV (256-383) and dK (384-511); the 64-query blocks are what lets
// two stages fit (an M = 128 tcgen05.mma costs about the same at N = 64 as at
// N = 128, but a single stage of 128-query tiles serialises the MMAs with the
// softmax-like P / dS work and measured slower).  The prep kernel also zeroes the
// dq accumulator.  Per block:
//   MMA   S^T, dP^T into the block's stage (issued two blocks ahead: S^T right
//         after the dV MMA of the block before in that stage, dP^T once that
//         block's dQ^T has been read out);
//   warps 4-11 (lane quarter = 32 keys, half = 32 queries) read S^T, dP^T, write
//         P^T as bf16 pairs over the first 16 of their S^T columns (the A operand
//         of the dV MMA) and dS into shared memory (K-major A of the dK MMA and
//         MN-major B of the dQ^T MMA);
//   MMA   dV += P^T dO, dK += dS^T Q, dQ^T = K^T dS^T over the stage's dP^T
//         columns (read into registers before the compute warps signalled);
//   warps 12-15 (one per lane quarter = 32 d) read dQ^T and add it into an fp32
//         accumulator in global memory, one 128-byte line per warp instruction
//         (reductions the L2 takes at its own rate, off the compute warps' path);
//         a last pass scales and rounds it (attn_dq_convert_kernel).
//   warp 0  TMA: K_j, V_j once, then Q, dO blocks (and L, D of their queries)
//           into a three-stage ring
//   warp 1  TMEM owner and MMA issuer
// The producer and the other warps wait suspended in mbarrier.try_wait (they
// share their schedulers with the MMA issuer, whose issue rate a spinning poll
// would take slots from); the issuer polls.  Every wait is bounded.
// ---------------------------------------------------------------------------
constexpr int kAbThreads = 512;
constexpr int kAbLaunchRegs = 128;  // 65536 / 512
// register split after setmaxnreg: producer / MMA warpgroup, two compute
// warpgroups, the dQ warpgroup (128 x 72 + 256 x 168 + 128 x 104 = 65536)
constexpr int kAbIssuerRegs = 72;
constexpr int kAbComputeRegs = 168;
constexpr int kAbReduceRegs = 104;
static_assert(128 * kAbIssuerRegs + 256 * kAbComputeRegs + 128 * kAbReduceRegs <= kAbThreads * kAbLaunchRegs,
              "register split");
constexpr int kAbBQ = 64;                   // queries per block
constexpr int kAbAtom = kAbBQ * 128;        // one 64-row x 64-column bf16 swizzle atom (8 KB)
constexpr int kAbBlock = 2 * kAbAtom;       // one 64 x 128 bf16 block (16 KB)
constexpr int kAbStages = 3;                // Q / dO ring
struct AbSmem {
  static constexpr int kK = 0;                          // K_j (K-major atoms, d 0-63 / 64-127)
  static constexpr int kV = kK + kAttTile;              // V_j
  static constexpr int kQ = kV + kAttTile;              // Q blocks, kAbStages stages
  static constexpr int kDO = kQ + kAbStages * kAbBlock; // dO blocks
  static constexpr int kDS = kDO + kAbStages * kAbBlock;  // dS per TMEM stage: [128 keys][64 queries], 128-byte swizzle
  static constexpr int kStats = kDS + 2 * kAbBlock;   // per Q / dO stage: L[64], D[64] fp32
  static constexpr int kStatBytes = 2 * kAbBQ * 4;
  static constexpr int kBars = kStats + kAbStages * kStatBytes;
  // kv_full, qd_full[3], qd_empty[3], s_full[2], pds_ready[2], dq_full[2], dq_free[2], dkv_done
  static constexpr int kNumBars = 16;
  static constexpr int kTmemSlot = kBars + kNumBars * 8;
  static constexpr int kBytes = kTmemSlot + 16;
};

struct AbParams {
  int B, T, H;
  int window;        // keys with t - k < window (window >= T: full causal)
  float scale;       // softmax scale
  float scale_log2;  // softmax scale * log2(e)
  const float* lse2; // [B, H, T] log-sum-exp in base 2 (lse log2 e)
  const float* Dv;   // [B, H, T] rowsum(dO . O)
  float* dq_acc;     // [B, T, H, 128] fp32, zeroed
  __nv_bfloat16* dk; // [B, T, H, 128]
  __nv_bfloat16* dv;
  int* err;
};

// D[b, h, t] = sum_d dO[b,t,h,d] O[b,t,h,d] and L[b, h, t] = lse[b, h, t] log2 e,
// and the row of the fp32 dq accumulator zeroed: one warp per (b, t, h) row.
__global__ void __launch_bounds__(256) attn_bwd_prep_kernel(const __nv_bfloat16* __restrict__ dout,
                                                            const __nv_bfloat16* __restrict__ out,
                                                            const float* __restrict__ lse, float* __restrict__ Dv,
                                                            float* __restrict__ lse2, float* __restrict__ dq_acc, int B,
                                                            int T, int H) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(B) * T * H;
  for (int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; row < rows;
       row += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const uint2 a = *reinterpret_cast<const uint2*>(dout + row * kAttD + 4 * lane);
    const uint2 o = *reinterpret_cast<const uint2*>(out + row * kAttD + 4 * lane);
    reinterpret_cast<float4*>(dq_acc + row * kAttD)[lane] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float acc = bf16_lo(a.x) * bf16_lo(o.x) + bf16_hi(a.x) * bf16_hi(o.x) + bf16_lo(a.y) * bf16_lo(o.y) +
                bf16_hi(a.y) * bf16_hi(o.y);
    acc = warp_sum(acc);
    if (lane == 0) {
      const int64_t bt = row / H;
      const int h = static_cast<int>(row - bt * H);
      const int64_t b = bt / T;
      const int64_t t = bt - b * T;
      const int64_t o = (b * H + h) * T + t;
      Dv[o] = acc;
      lse2[o] = lse[o] * 1.4426950408889634f;
    }
  }
}

// dq = bf16(scale * dq_acc)
__global__ void __launch_bounds__(256) attn_dq_convert_kernel(const float* __restrict__ acc, float scale,
                                                              __nv_bfloat16* __restrict__ dq, int64_t n4) {
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < n4;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 x = reinterpret_cast<const float4*>(acc)[v];
    uint2 o;
    o.x = pack_bf16x2(x.x * scale, x.y * scale);
    o.y = pack_bf16x2(x.z * scale, x.w * scale);
    reinterpret_cast<uint2*>(dq)[v] = o;
  }
}

HLM_DEVICE void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// P^T = 2^(S^T sc - L) and dS^T = P^T (dP^T - D) of one key row over 32 queries,
// packed as bf16 query pairs; L and D are the shared-memory addresses of the first
// query's entries (every lane reads the same 16 bytes), dq0 = first query - key
// (the pair is kept when 0 <= q - key < window).
template <bool kMask>
__device__ __forceinline__ void ab_p_ds(const uint32_t (&sx)[32], const uint32_t (&dpx)[32], uint32_t (&pk)[16],
                                        uint32_t (&dk2)[16], uint32_t L, uint32_t D, int dq0, int window, float sc) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const uint4 l4 = ld_shared_v4(L + static_cast<uint32_t>(i * 4));
    const uint4 d4 = ld_shared_v4(D + static_cast<uint32_t>(i * 4));
    const float lq[4] = {__uint_as_float(l4.x), __uint_as_float(l4.y), __uint_as_float(l4.z), __uint_as_float(l4.w)};
    const float dq[4] = {__uint_as_float(d4.x), __uint_as_float(d4.y), __uint_as_float(d4.z), __uint_as_float(d4.w)};
    float pv[4], dsv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float pq = ex2_ftz(fmaf(__uint_as_float(sx[i + e]), sc, -lq[e]));
      if (kMask) {
        const int d = dq0 + i + e;
        pq = (d >= 0 && d < window) ? pq : 0.0f;
      }
      pv[e] = pq;
      dsv[e] = pq * (__uint_as_float(dpx[i + e]) - dq[e]);
    }
    pk[i / 2] = pack_bf16x2(pv[0], pv[1]);
    pk[i / 2 + 1] = pack_bf16x2(pv[2], pv[3]);
    dk2[i / 2] = pack_bf16x2(dsv[0], dsv[1]);
    dk2[i / 2 + 1] = pack_bf16x2(dsv[2], dsv[3]);
  }
}

// One block's dQ^T column slice (this thread's d, 32 queries qstride apart) added
// into the fp32 accumulator.
HLM_DEVICE void ab_dq_reduce(float* dst, int64_t qstride, const uint32_t (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i)
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(dst + i * qstride), "f"(__uint_as_float(v[i])) : "memory");
}

__global__ void __launch_bounds__(kAbThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const AbParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = p.err;

  // work item: key tile j of one (b, h), key tiles in increasing order over the
  // grid (the lowest see the most query blocks under the causal mask)
  const int BH = p.B * p.H;
  const int j = static_cast<int>(blockIdx.x) / BH;
  const int bh = static_cast<int>(blockIdx.x) - j * BH;
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  // query blocks qb0 .. qb_last: query q sees a key of tile j while
  // 0 <= q - k < window for some k in [128 j, 128 j + 127]
  const int qb0 = j * (kAttBK / kAbBQ);
  const int qb_last = min(p.T / kAbBQ - 1, (j * kAttBK + kAttBK - 2 + p.window) / kAbBQ);
  const int n_i = qb_last - qb0 + 1;

  const uint32_t bar0 = base + AbSmem::kBars;
  const uint32_t kv_full = bar0;
  auto qd_full = [&](int s) { return bar0 + 8u * static_cast<uint32_t>(1 + s); };
  auto qd_empty = [&](int s) { return bar0 + 8u * static_cast<uint32_t>(4 + s); };
  auto s_full = [&](int st) { return bar0 + 8u * static_cast<uint32_t>(7 + st); };
  auto pds_ready = [&](int st) { return bar0 + 8u * static_cast<uint32_t>(9 + st); };
  auto dq_full = [&](int st) { return bar0 + 8u * static_cast<uint32_t>(11 + st); };
  auto dq_free = [&](int st) { return bar0 + 8u * static_cast<uint32_t>(13 + st); };
  const uint32_t dkv_done = bar0 + 8u * 15u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + AbSmem::kTmemSlot);

  if (warp == 0 && lane == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < kAbStages; ++s) {
      mbar_init(qd_full(s), 1);
      mbar_init(qd_empty(s), 1);
    }
    for (int st = 0; st < 2; ++st) {
      mbar_init(s_full(st), 1);
      mbar_init(pds_ready(st), 8);
      mbar_init(dq_full(st), 1);
      mbar_init(dq_free(st), 4);
    }
    mbar_init(dkv_done, 1);
    fence_mbar_init();
    prefetch_tensormap(&tmQ);
    prefetch_tensormap(&tmK);
    prefetch_tensormap(&tmV);
    prefetch_tensormap(&tmDO);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // stage st: S^T (then P^T over its first columns) at 128 st, dP^T (then the
  // block's dQ^T) at 128 st + 64
  auto t_stage = [&](int st) { return tmem_base + 128u * static_cast<uint32_t>(st); };
  const uint32_t t_dv = tmem_base + 256u, t_dk = tmem_base + 384u;
  const int row_k = b * p.T + j * kAttBK;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kAbIssuerRegs));
  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, 2 * kAttTile);
      for (int a = 0; a < 2; ++a) {
        tma_load_2d(base + AbSmem::kK + static_cast<uint32_t>(a * kAttAtom), &tmK, h * kAttD + 64 * a, row_k, kv_full);
        tma_load_2d(base + AbSmem::kV + static_cast<uint32_t>(a * kAttAtom), &tmV, h * kAttD + 64 * a, row_k, kv_full);
      }
      int issued = 0;
      for (int ii = 0; ii < n_i; ++ii) {
        const int s = ii % kAbStages;
        if (ii >= kAbStages &&
            !mbar_wait(qd_empty(s), static_cast<uint32_t>((ii / kAbStages - 1) & 1), err, kDevErrTimeoutEmpty))
          break;
        const int row_q = b * p.T + (qb0 + ii) * kAbBQ;
        const int64_t stat = static_cast<int64_t>(bh) * p.T + (qb0 + ii) * kAbBQ;
        const uint32_t stats = base + AbSmem::kStats + static_cast<uint32_t>(s * AbSmem::kStatBytes);
        mbar_arrive_expect_tx(qd_full(s), 2 * kAbBlock + AbSmem::kStatBytes);
        bulk_load_1d(stats, p.lse2 + stat, kAbBQ * 4, qd_full(s));
        bulk_load_1d(stats + kAbBQ * 4, p.Dv + stat, kAbBQ * 4, qd_full(s));
        for (int a = 0; a < 2; ++a) {
          tma_load_2d(base + AbSmem::kQ + static_cast<uint32_t>(s * kAbBlock + a * kAbAtom), &tmQ, h * kAttD + 64 * a,
                      row_q, qd_full(s));
          tma_load_2d(base + AbSmem::kDO + static_cast<uint32_t>(s * kAbBlock + a * kAbAtom), &tmDO,
                      h * kAttD + 64 * a, row_q, qd_full(s));
        }
        issued = ii + 1;
      }
      mbar_wait_drain(kv_full, 0u, err);
      for (int ii = max(0, issued - kAbStages); ii < issued; ++ii)
        mbar_wait_drain(qd_full(ii % kAbStages), static_cast<uint32_t>((ii / kAbStages) & 1), err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, kAbBQ, false, false);  // S^T, dP^T
      constexpr uint32_t idesc_kv = make_idesc_bf16_f32(128, 128, false, true);    // dV (A in TMEM), dK
      constexpr uint32_t idesc_q = make_idesc_bf16_f32(128, kAbBQ, true, true);    // dQ^T
      const uint64_t dk_kmaj = make_sw128_desc(base + AbSmem::kK, 16u, 1024u);
      const uint64_t dv_kmaj = make_sw128_desc(base + AbSmem::kV, 16u, 1024u);
      const uint64_t dk_mn = make_sw128_desc(base + AbSmem::kK, kAttAtom, 1024u);
      // S^T = K Q^T and dP^T = V dO^T of block ii into its stage, once the block
      // two before it (same stage) has had its dQ^T read out
      // S^T = K Q^T of block ii into its stage's S^T columns (descriptors advance by
      // the operand offset / 16: the address field, no carry out of it inside
      // shared memory); the block's Q / dO stage must have landed
      auto issue_s = [&](int ii) -> bool {
        const int s = ii % kAbStages;
        if (!mbar_poll(qd_full(s), static_cast<uint32_t>((ii / kAbStages) & 1), err, kDevErrTimeoutFull)) return false;
        tc_fence_after();
        const uint64_t dq_ = make_sw128_desc(base + AbSmem::kQ + static_cast<uint32_t>(s * kAbBlock), 16u, 1024u);
#pragma unroll
        for (int kk = 0; kk < kAttD / kUmmaK; ++kk)
          tc_mma_f16(t_stage(ii & 1), dk_kmaj + ((kk >> 2) * kAttAtom + (kk & 3) * 32) / 16,
                     dq_ + ((kk >> 2) * kAbAtom + (kk & 3) * 32) / 16, idesc_s, kk > 0 ? 1u : 0u);
        return true;
      };
      // dP^T = V dO^T of block ii into its stage's dP^T columns, then publish the stage
      auto issue_dp = [&](int ii) {
        const int s = ii % kAbStages;
        const uint64_t ddo = make_sw128_desc(base + AbSmem::kDO + static_cast<uint32_t>(s * kAbBlock), 16u, 1024u);
#pragma unroll
        for (int kk = 0; kk < kAttD / kUmmaK; ++kk)
          tc_mma_f16(t_stage(ii & 1) + 64u, dv_kmaj + ((kk >> 2) * kAttAtom + (kk & 3) * 32) / 16,
                     ddo + ((kk >> 2) * kAbAtom + (kk & 3) * 32) / 16, idesc_s, kk > 0 ? 1u : 0u);
        tc_commit(s_full(ii & 1));
      };
      bool ok = mbar_poll(kv_full, 0u, err, kDevErrTimeoutFull);
      for (int ii = 0; ii < 2 && ii < n_i && ok; ++ii)
        if ((ok = issue_s(ii))) issue_dp(ii);
      for (int ii = 0; ii < n_i && ok; ++ii) {
        const int s = ii % kAbStages, st = ii & 1;
        if (!(ok = mbar_poll(pds_ready(st), static_cast<uint32_t>((ii >> 1) & 1), err, kDevErrTimeoutFull))) break;
        tc_fence_after();
        const uint32_t qbase = base + AbSmem::kQ + static_cast<uint32_t>(s * kAbBlock);
        const uint32_t dobase = base + AbSmem::kDO + static_cast<uint32_t>(s * kAbBlock);
        const uint32_t dsbase = base + AbSmem::kDS + static_cast<uint32_t>(st * kAbBlock);
        const uint64_t ddo_mn = make_sw128_desc(dobase, kAbAtom, 1024u);
        const uint64_t dq_mn = make_sw128_desc(qbase, kAbAtom, 1024u);
        const uint64_t dds_k = make_sw128_desc(dsbase, 16u, 1024u);
        const uint64_t dds_mn = make_sw128_desc(dsbase, kAbBlock, 1024u);
        // dV += P^T dO: A = P^T from TMEM (16 queries per step: half kk >> 1 of the
        // block, 8 packed columns in), B = dO as MN-major (d contiguous, the two
        // 64-wide d atoms 8 KB apart, 16 query rows per step)
#pragma unroll
        for (int kk = 0; kk < kAbBQ / kUmmaK; ++kk)
          tc_mma_f16_ts(t_dv, t_stage(st) + static_cast<uint32_t>((kk >> 1) * 32 + (kk & 1) * 8), ddo_mn + kk * 2048 / 16,
                        idesc_kv, (ii > 0 || kk > 0) ? 1u : 0u);
        // dK += dS^T Q: A = dS as K-major (keys are rows, queries contiguous), B = Q as MN-major
#pragma unroll
        for (int kk = 0; kk < kAbBQ / kUmmaK; ++kk)
          tc_mma_f16(t_dk, dds_k + kk * 32 / 16, dq_mn + kk * 2048 / 16, idesc_kv, (ii > 0 || kk > 0) ? 1u : 0u);
        // dQ^T = K^T dS^T over the stage's dP^T columns (read into registers before
        // pds_ready): A = K as MN-major (d contiguous, the two d atoms 16 KB apart),
        // B = dS as MN-major (queries contiguous), 16 keys per step
#pragma unroll
        for (int kk = 0; kk < kAttBK / kUmmaK; ++kk)
          tc_mma_f16(t_stage(st) + 64u, dk_mn + kk * 2048 / 16, dds_mn + kk * 2048 / 16, idesc_q, kk > 0 ? 1u : 0u);
        tc_commit(dq_full(st));
        tc_commit(qd_empty(s));
        // block ii + 2 into this stage: S^T right behind the dV MMA that read P^T
        // from those columns (one thread's MMAs run in order), dP^T once this
        // block's dQ^T has been read out
        if (ii + 2 < n_i) {
          if (!(ok = issue_s(ii + 2))) break;
          if (!(ok = mbar_poll(dq_free(st), static_cast<uint32_t>((ii >> 1) & 1), err, kDevErrTimeoutTmemEmpty))) break;
          tc_fence_after();
          issue_dp(ii + 2);
        }
      }
      if (ok) tc_commit(dkv_done);
    }
  }
  } else if (warp < 12) {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kAbComputeRegs));
    const int quad = warp & 3;          // TMEM lane quarter
    const int hh = (warp - 4) >> 2;     // half of the block's queries: 32 hh .. 32 hh + 31
    const int kr = quad * 32 + lane;    // key row of the tile (and d of the dQ^T lanes)
    const int key = j * kAttBK + kr;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float sc = p.scale_log2;
    bool ok = true;
    for (int ii = 0; ii < n_i; ++ii) {
      const int st = ii & 1;
      const uint32_t par = static_cast<uint32_t>((ii >> 1) & 1);
      const int q0 = (qb0 + ii) * kAbBQ + 32 * hh;  // first query of this warp's columns
      // S^T, dP^T in TMEM; L, D of the block in its Q / dO stage (that TMA phase
      // completed before the MMA thread issued S^T)
      if (!warp_wait(s_full(st), par, err, kDevErrTimeoutTmemFull, lane) ||
          !warp_wait(qd_full(ii % kAbStages), static_cast<uint32_t>((ii / kAbStages) & 1), err, kDevErrTimeoutFull,
                     lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sx[32], dpx[32];
      tmem_ld_32x32b_x32(t_stage(st) + lane_off + static_cast<uint32_t>(32 * hh), sx);
      tmem_ld_32x32b_x32(t_stage(st) + lane_off + static_cast<uint32_t>(64 + 32 * hh), dpx);
      tmem_ld_wait();
      // P^T and dS^T for queries q0 .. q0 + 31 (masked pairs give 0; only the two
      // diagonal blocks and the blocks the window edge crosses hold any)
      uint32_t pk[16], dk2[16];
      const uint32_t stats =
          base + AbSmem::kStats + static_cast<uint32_t>((ii % kAbStages) * AbSmem::kStatBytes + 32 * hh * 4);
      if (ii < kAttBK / kAbBQ || (qb0 + ii) * kAbBQ + kAbBQ - 1 - j * kAttBK >= p.window)
        ab_p_ds<true>(sx, dpx, pk, dk2, stats, stats + kAbBQ * 4, q0 - key, p.window, sc);
      else
        ab_p_ds<false>(sx, dpx, pk, dk2, stats, stats + kAbBQ * 4, q0 - key, p.window, sc);
      // P^T pairs over the first 16 of the 32 S^T columns this warp read (the other
      // warp of the lane quarter reads the other 32); dS into this stage's shared
      // buffer (row = key, 64 queries, 128-byte swizzle; this warp's 32 queries are
      // 16-byte chunks 4 hh .. 4 hh + 3), which the block two before released (its
      // dK and dQ^T MMAs completed before this block's dP^T was issued)
      tmem_st_32x32b_x16(t_stage(st) + lane_off + static_cast<uint32_t>(32 * hh), pk);
      const uint32_t ds_row = base + AbSmem::kDS + static_cast<uint32_t>(st * kAbBlock + kr * 128);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        st_shared_v4(ds_row + static_cast<uint32_t>(((4 * hh + c) ^ (kr & 7)) << 4),
                     make_uint4(dk2[4 * c], dk2[4 * c + 1], dk2[4 * c + 2], dk2[4 * c + 3]));
      fence_proxy_async_smem();
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(pds_ready(st));
    }
    // dK (scaled) and dV of this key tile: TMEM lanes = keys, columns = d 64 hh ..
    if (ok && warp_wait(dkv_done, 0u, err, kDevErrTimeoutTmemFull, lane)) {
      tc_fence_after();
      const int64_t o = (static_cast<int64_t>(b * p.T + key) * p.H + h) * kAttD + 64 * hh;
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        uint32_t x[2][32];
        const uint32_t t = (which == 0 ? t_dk : t_dv) + lane_off + static_cast<uint32_t>(64 * hh);
        tmem_ld_32x32b_x32(t, x[0]);
        tmem_ld_32x32b_x32(t + 32u, x[1]);
        tmem_ld_wait();
        const float f = which == 0 ? p.scale : 1.0f;
        __nv_bfloat16* d = (which == 0 ? p.dk : p.dv) + o;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int i = 0; i < 32; i += 8)
            st_global_v4(d + 32 * c + i,
                         make_uint4(pack_bf16x2(__uint_as_float(x[c][i]) * f, __uint_as_float(x[c][i + 1]) * f),
                                    pack_bf16x2(__uint_as_float(x[c][i + 2]) * f, __uint_as_float(x[c][i + 3]) * f),
                                    pack_bf16x2(__uint_as_float(x[c][i + 4]) * f, __uint_as_float(x[c][i + 5]) * f),
                                    pack_bf16x2(__uint_as_float(x[c][i + 6]) * f, __uint_as_float(x[c][i + 7]) * f)));
      }
    }
  } else {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kAbReduceRegs));
    // each block's dQ^T: TMEM lanes = d 32 quad .., dP^T columns = its 64 queries
    const int quad = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int64_t qstride = static_cast<int64_t>(p.H) * kAttD;
    for (int ii = 0; ii < n_i; ++ii) {
      const int st = ii & 1;
      if (!warp_wait(dq_full(st), static_cast<uint32_t>((ii >> 1) & 1), err, kDevErrTimeoutTmemFull, lane)) break;
      tc_fence_after();
      uint32_t dq[2][32];
      tmem_ld_32x32b_x32(t_stage(st) + lane_off + 64u, dq[0]);
      tmem_ld_32x32b_x32(t_stage(st) + lane_off + 96u, dq[1]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free(st));
      float* dst = p.dq_acc + (static_cast<int64_t>(b * p.T + (qb0 + ii) * kAbBQ) * p.H + h) * kAttD + quad * 32 + lane;
      ab_dq_reduce(dst, qstride, dq[0]);
      ab_dq_reduce(dst + 32 * qstride, qstride, dq[1]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}
}  // namespace hlm

using namespace hlm;

extern "C" int hlm_attention_fwd(const void* q, const void* k, const void* v, void* out, float* lse, int64_t B,
                                 int64_t T, int64_t H, int64_t Hk, int64_t D, int64_t window, float scale,
                                 void* stream) {
  if (B < 0 || T < 0 || H <= 0 || Hk <= 0 || D <= 0) return HLM_ERR_INVALID_ARG;
  if (B == 0 || T == 0) return HLM_OK;
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr || lse == nullptr) return HLM_ERR_INVALID_ARG;
  if (D != kAttD || T % kAttBQ != 0 || H % Hk != 0) return HLM_ERR_UNSUPPORTED;
  if (B * T > (1ll << 30) || B * H * (T / kAttBQ) > (1ll << 30)) return HLM_ERR_UNSUPPORTED;
  const void* ptrs[] = {q, k, v, out};
  for (const void* ptr : ptrs)
    if (!host_aligned16(ptr)) return HLM_ERR_UNSUPPORTED;
  CUtensorMap mq, mk, mv, mo;
  const int64_t rows = B * T;
  if (!encode_bf16_map(&mq, q, H * D, rows, H * D, 128) || !encode_bf16_map(&mk, k, Hk * D, rows, Hk * D, 128) ||
      !encode_bf16_map(&mv, v, Hk * D, rows, Hk * D, 64) || !encode_bf16_map(&mo, out, H * D, rows, H * D, 32))
    return HLM_ERR_DRIVER;
  AttParams p;
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.Hk = static_cast<int>(Hk);
  p.window = window <= 0 || window >= T ? static_cast<int>(T) : static_cast<int>(window);
  p.q_tiles = static_cast<int>(T / kAttBQ);
  p.q_pairs = (p.q_tiles + 1) / 2;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse = lse;
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  const int smem = AttSmem::kBytes + 1024;
  static_assert(AttSmem::kBytes + 1024 <= 232448, "shared memory budget exceeded");
  if (cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  static const int compiled_regs = [] {
    cudaFuncAttributes attr{};
    return cudaFuncGetAttributes(&attr, attn_fwd_kernel) == cudaSuccess ? attr.numRegs : -1;
  }();
  if (compiled_regs != kAttLaunchRegs) return HLM_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t grid = B * H * p.q_pairs;
  {
    LaunchScope scope(HLM_KERNEL_ATTN_FWD, s);
    attn_fwd_kernel<<<static_cast<unsigned>(grid), kAttThreads, smem, s>>>(mq, mk, mv, mo, p);
  }
  return launch_status();
}

extern "C" size_t hlm_attention_bwd_workspace_bytes(int64_t B, int64_t T, int64_t H, int64_t D) {
  if (B <= 0 || T <= 0 || H <= 0 || D <= 0) return 0;
  return static_cast<size_t>(B * T * H * D) * 4 + static_cast<size_t>(B * H * T) * 8 + 256;
}

extern "C" int hlm_attention_bwd(const void* grad_out, const void* q, const void* k, const void* v, const void* out,
                                 const float* lse, void* dq, void* dk, void* dv, void* workspace,
                                 size_t workspace_bytes, int64_t B, int64_t T, int64_t H, int64_t Hk, int64_t D,
                                 int64_t window, float scale, void* stream) {
  if (B < 0 || T < 0 || H <= 0 || Hk <= 0 || D <= 0) return HLM_ERR_INVALID_ARG;
  if (B == 0 || T == 0) return HLM_OK;
  const void* ptrs[] = {grad_out, q, k, v, out, lse, dq, dk, dv, workspace};
  for (const void* ptr : ptrs)
    if (ptr == nullptr) return HLM_ERR_INVALID_ARG;
  if (D != kAttD || T % kAttBQ != 0 || Hk != H) return HLM_ERR_UNSUPPORTED;
  if (B * T * H > (1ll << 30)) return HLM_ERR_UNSUPPORTED;
  for (const void* ptr : ptrs)
    if (!host_aligned16(ptr)) return HLM_ERR_UNSUPPORTED;
  if (workspace_bytes < hlm_attention_bwd_workspace_bytes(B, T, H, D)) return HLM_ERR_INVALID_ARG;
  float* dq_acc = static_cast<float*>(workspace);
  float* Dv = dq_acc + B * T * H * D;
  float* lse2 = Dv + B * H * T;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int sms = num_sms_of_current_device();
  {
    const int64_t rows = B * T * H;
    int64_t blocks = (rows * 32 + 255) / 256;
    if (blocks > static_cast<int64_t>(sms) * 8) blocks = static_cast<int64_t>(sms) * 8;
    LaunchScope scope(HLM_KERNEL_ATTN_BWD, s);
    attn_bwd_prep_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(grad_out), static_cast<const __nv_bfloat16*>(out), lse, Dv, lse2, dq_acc,
        static_cast<int>(B),
        static_cast<int>(T), static_cast<int>(H));
  }
  if (launch_status() != HLM_OK) return HLM_ERR_LAUNCH;
  CUtensorMap mq, mk, mv, mdo;
  const int64_t rows = B * T;
  if (!encode_bf16_map(&mq, q, H * D, rows, H * D, kAbBQ) || !encode_bf16_map(&mk, k, H * D, rows, H * D, 128) ||
      !encode_bf16_map(&mv, v, H * D, rows, H * D, 128) || !encode_bf16_map(&mdo, grad_out, H * D, rows, H * D, kAbBQ))
    return HLM_ERR_DRIVER;
  AbParams p;
  p.B = static_cast<int>(B);
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.window = window <= 0 || window >= T ? static_cast<int>(T) : static_cast<int>(window);
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse2 = lse2;
  p.Dv = Dv;
  p.dq_acc = dq_acc;
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  const int smem = AbSmem::kBytes + 1024;
  static_assert(AbSmem::kBytes + 1024 <= 232448, "shared memory budget exceeded");
  if (cudaFuncSetAttribute(attn_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  static const int compiled_regs = [] {
    cudaFuncAttributes attr{};
    return cudaFuncGetAttributes(&attr, attn_bwd_kernel) == cudaSuccess ? attr.numRegs : -1;
  }();
  if (compiled_regs != kAbLaunchRegs) return HLM_ERR_UNSUPPORTED;
  {
    LaunchScope scope(HLM_KERNEL_ATTN_BWD, s);
    attn_bwd_kernel<<<static_cast<unsigned>(B * H * (T / kAttBK)), kAbThreads, smem, s>>>(mq, mk, mv, mdo, p);
  }
  if (launch_status() != HLM_OK) return HLM_ERR_LAUNCH;
  {
    const int64_t n4 = B * T * H * D / 4;
    int64_t blocks = (n4 + 255) / 256;
    if (blocks > static_cast<int64_t>(sms) * 8) blocks = static_cast<int64_t>(sms) * 8;
    LaunchScope scope(HLM_KERNEL_ATTN_BWD, s);
    attn_dq_convert_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(dq_acc, scale, static_cast<__nv_bfloat16*>(dq), n4);
  }
  return launch_status();
}
