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
// One CTA takes 128 query rows of one (b, h) and walks the key tiles of 128 from
// the first the window reaches to the diagonal:
//   warp 0  TMA producer: Q once, then K_j / V_j into a two-stage ring
//   warp 1  TMEM owner and MMA issuer: S_j = Q K_j^T (M=N=K=128) into one of two
//           TMEM score buffers, issued one tile ahead; O += P_j V_j into the TMEM
//           output accumulator once the softmax warps have written P_j
//   warps 2-5  softmax, one query row per thread: the score row into registers
//           (one read of the score buffer), row max and exp2 of the scaled, masked
//           scores against a reference max that moves only when a tile exceeds it
//           by more than 8, running sum, P_j as bf16 into shared memory (the
//           128-byte-swizzled K-major layout of the PV MMA's A operand), and, on a
//           move, the output row rescaled in TMEM (tcgen05.ld / st) before PV_j; at
//           the end out = O / l through TMA stores and lse = (m + log2 l) ln 2.
// P_j is written only after PV_{j-1} has finished reading the single P buffer and
// updating O; S_{j+1} runs on the tensor cores meanwhile.  Every wait is bounded.
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

// Waits on the per-tile chain (S -> softmax -> P -> PV -> next P) poll the barrier
// with mbarrier.test_wait instead of suspending in try_wait: every one of them is
// on the critical path, and a suspended thread resumes late (measured: 10x slower
// with suspending waits).  Bounded like every other wait.
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
// `backoff_ns` > 0: sleep that long between polls, for the single-thread roles
// (producer, MMA issuer) whose warps share a scheduler with a softmax warp.
HLM_DEVICE bool mbar_poll(uint32_t bar, uint32_t parity, int* err, int code, uint32_t backoff_ns = 0) {
  if (mbar_test(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (backoff_ns) __nanosleep(backoff_ns);
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

constexpr int kAttD = 128;         // head dim
constexpr int kAttBQ = 128;        // query rows per CTA
constexpr int kAttBK = 128;        // keys per tile
constexpr int kAttStages = 2;      // K/V ring
constexpr int kAttAtom = 128 * 128;  // one 128-row x 64-column bf16 swizzle atom (16 KB)

struct AttSmem {
  static constexpr int kQ = 0;                            // 2 atoms (d 0-63, 64-127)
  static constexpr int kKV = kQ + 2 * kAttAtom;           // per stage: K 2 atoms, V 2 key blocks x 2 d blocks
  static constexpr int kStageBytes = 4 * kAttAtom;        // 64 KB
  static constexpr int kP = kKV + kAttStages * kStageBytes;  // 2 atoms (keys 0-63, 64-127)
  static constexpr int kBars = kP + 2 * kAttAtom;
  // barriers: q_full, kv_full[2], kv_empty[2], s_full[2], s_empty[2], p_full, pv_done
  static constexpr int kNumBars = 11;
  static constexpr int kTmemSlot = kBars + kNumBars * 8;
  static constexpr int kBytes = kTmemSlot + 16;
};

struct AttParams {
  int B, T, H, Hk;
  int window;       // keys with t - k < window (window >= T: full causal)
  int q_tiles;      // T / 128
  float scale_log2; // softmax scale * log2(e)
  float* lse;       // [B, H, T]
  int* err;
};

__global__ void __launch_bounds__(192, 1)
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

  // work item: longest (highest) query tiles first
  const int per_bh = p.q_tiles;
  const int item = static_cast<int>(blockIdx.x);
  const int bh = item / per_bh;
  const int qi = per_bh - 1 - (item - bh * per_bh);
  const int b = bh / p.H;
  const int h = bh - b * p.H;
  const int hk = h / (p.H / p.Hk);
  const int q0 = qi * kAttBQ;
  const int first_key = max(0, q0 - p.window + 1);
  const int j0 = first_key / kAttBK;
  const int nt = qi - j0 + 1;  // key tiles j0 .. qi

  const uint32_t bar0 = base + AttSmem::kBars;
  const uint32_t q_full = bar0;
  auto kv_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto kv_empty = [&](int s) { return bar0 + 8u * (3 + s); };
  auto s_full = [&](int s) { return bar0 + 8u * (5 + s); };
  auto s_empty = [&](int s) { return bar0 + 8u * (7 + s); };
  const uint32_t p_full = bar0 + 8u * 9;
  const uint32_t pv_done = bar0 + 8u * 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base_ptr + AttSmem::kTmemSlot);

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
      mbar_init(s_full(s), 1);
      mbar_init(s_empty(s), 4);  // the four softmax warps
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
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
  const uint32_t t_s[2] = {tmem_base, tmem_base + 128u};
  const uint32_t t_o = tmem_base + 256u;
  const int row_q = b * p.T + q0;         // first query row in the [B*T, H*D] view
  const int row_k0 = b * p.T;             // first key row of this sequence

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(q_full, 2 * kAttAtom);
      tma_load_2d(base + AttSmem::kQ, &tmQ, h * kAttD, row_q, q_full);
      tma_load_2d(base + AttSmem::kQ + kAttAtom, &tmQ, h * kAttD + 64, row_q, q_full);
      uint32_t armed = 0, armed_par = 0;
      for (int t = 0; t < nt && ok; ++t) {
        const int s = t & 1;
        if (t >= 2 && !mbar_poll(kv_empty(s), static_cast<uint32_t>(((t >> 1) - 1) & 1), err, kDevErrTimeoutEmpty, 64)) {
          ok = false;
          break;
        }
        const uint32_t st = base + AttSmem::kKV + static_cast<uint32_t>(s * AttSmem::kStageBytes);
        const int key0 = row_k0 + (j0 + t) * kAttBK;
        mbar_arrive_expect_tx(kv_full(s), AttSmem::kStageBytes);
        armed |= 1u << s;
        armed_par = (armed_par & ~(1u << s)) | ((static_cast<uint32_t>(t >> 1) & 1u) << s);
        // K: two K-major atoms [128 keys][64 d]
        tma_load_2d(st, &tmK, hk * kAttD, key0, kv_full(s));
        tma_load_2d(st + kAttAtom, &tmK, hk * kAttD + 64, key0, kv_full(s));
        // V: MN-major blocks [64 keys][64 d]: key block kb at 16 KB, d block i at 8 KB
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int i = 0; i < 2; ++i)
            tma_load_2d(st + 2 * kAttAtom + static_cast<uint32_t>(kb * 16384 + i * 8192), &tmVk, hk * kAttD + 64 * i,
                        key0 + 64 * kb, kv_full(s));
      }
      for (int s = 0; s < 2; ++s)
        if (armed & (1u << s)) mbar_wait_drain(kv_full(s), (armed_par >> s) & 1u, err);
      mbar_wait_drain(q_full, 0u, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, 128, false, true);
      bool ok = mbar_poll(q_full, 0u, err, kDevErrTimeoutFull, 32);
      auto issue_s = [&](int t) -> bool {
        const int s = t & 1;
        if (!mbar_poll(kv_full(s), static_cast<uint32_t>((t >> 1) & 1), err, kDevErrTimeoutFull, 32)) return false;
        if (t >= 2 && !mbar_poll(s_empty(s), static_cast<uint32_t>(((t >> 1) - 1) & 1), err, kDevErrTimeoutTmemEmpty, 32))
          return false;
        tc_fence_after();
        const uint32_t sk = base + AttSmem::kKV + static_cast<uint32_t>(s * AttSmem::kStageBytes);
#pragma unroll
        for (int kk = 0; kk < kAttD / kUmmaK; ++kk) {
          const uint32_t atom = static_cast<uint32_t>((kk >> 2) * kAttAtom + (kk & 3) * 32);
          tc_mma_f16(t_s[s], make_sw128_desc(base + AttSmem::kQ + atom, 16u, 1024u),
                     make_sw128_desc(sk + atom, 16u, 1024u), idesc_s, kk > 0 ? 1u : 0u);
        }
        tc_commit(s_full(s));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int t = 0; t < nt && ok; ++t) {
        if (t + 1 < nt && !(ok = issue_s(t + 1))) break;
        if (!mbar_poll(p_full, static_cast<uint32_t>(t & 1), err, kDevErrTimeoutFull, 32)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int s = t & 1;
        const uint32_t sv = base + AttSmem::kKV + static_cast<uint32_t>(s * AttSmem::kStageBytes + 2 * kAttAtom);
#pragma unroll
        for (int kk = 0; kk < kAttBK / kUmmaK; ++kk) {
          // A = P [128 q][128 keys] K-major (two 64-key atoms); B = V MN-major
          const uint32_t pa = base + AttSmem::kP + static_cast<uint32_t>((kk >> 2) * kAttAtom + (kk & 3) * 32);
          const uint32_t vb = sv + static_cast<uint32_t>((kk >> 2) * 16384 + (kk & 3) * 2048);
          tc_mma_f16(t_o, make_sw128_desc(pa, 16u, 1024u), make_sw128_desc(vb, 8192u, 1024u), idesc_o,
                     (t > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(kv_empty(s));
        tc_commit(pv_done);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // row of the tile
    const int qpos = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float sc = p.scale_log2;
    float m = -INFINITY, l = 0.0f;  // reference max (log2 domain) and row sum
    bool ok = true;
    for (int t = 0; t < nt; ++t) {
      const int s = t & 1;
      const int key0 = (j0 + t) * kAttBK;
      if (!warp_poll(s_full(s), static_cast<uint32_t>((t >> 1) & 1), err, kDevErrTimeoutTmemFull, lane)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // the whole score row into registers (four loads, one wait), which frees the
      // score buffer for S_{t+2}
      const bool full_tile = key0 + kAttBK - 1 <= q0 && q0 + kAttBQ - 1 - key0 < p.window;
      uint32_t x[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_s[s] + lane_off + static_cast<uint32_t>(c * 32), x[c]);
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty(s));
      // scaled, masked scores (log2 domain) and their row max (eight independent
      // partial maxima / sums: the reductions would otherwise be one dependent chain)
      float mxp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mxp[u] = -INFINITY;
      if (full_tile) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float v = __uint_as_float(x[c][i]) * sc;
            x[c][i] = __float_as_uint(v);
            mxp[i & 7] = fmaxf(mxp[i & 7], v);
          }
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int key = key0 + c * 32 + i;
            const bool valid = key <= qpos && qpos - key < p.window;
            const float v = valid ? __uint_as_float(x[c][i]) * sc : -INFINITY;
            x[c][i] = __float_as_uint(v);
            mxp[i & 7] = fmaxf(mxp[i & 7], v);
          }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                             fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
      // The exponent's reference max moves only when this tile exceeds it by more
      // than 8 (so p <= 256): softmax does not depend on the reference, and O and l
      // are rescaled (alpha) only on those moves.  alpha is 0 when the row had no
      // valid key before (its O row and l are 0).
      float alpha = 1.0f;
      if (mx > m + 8.0f) {
        alpha = ex2_ftz(m - mx);
        m = mx;
      }
      const float m_use = m == -INFINITY ? 0.0f : m;
      // p = exp2(s - m) packed to bf16 for the PV MMA; the row sum (and so the
      // log-sum-exp the backward recomputes P from) takes the fp32 values
      uint32_t pk[64];
      float rsp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) rsp[u] = 0.0f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float e0 = ex2_ftz(__uint_as_float(x[c][i]) - m_use);
          const float e1 = ex2_ftz(__uint_as_float(x[c][i + 1]) - m_use);
          rsp[(i >> 1) & 7] += e0 + e1;
          pk[c * 16 + i / 2] = pack_bf16x2(e0, e1);
        }
      }
      const float rs = ((rsp[0] + rsp[1]) + (rsp[2] + rsp[3])) + ((rsp[4] + rsp[5]) + (rsp[6] + rsp[7]));
      l = alpha * l + rs;
      // PV_{t-1} done: the P buffer is free and O holds the sum up to t-1
      if (t > 0) {
        if (!warp_poll(pv_done, static_cast<uint32_t>((t - 1) & 1), err, kDevErrTimeoutTmemFull, lane)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // P row -> shared memory: key chunk k (8 keys = 16 bytes) of atom k / 8
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        const uint32_t addr = base + AttSmem::kP + static_cast<uint32_t>((k >> 3) * kAttAtom + r * 128 +
                                                                          (((k & 7) ^ (r & 7)) << 4));
        st_shared_v4(addr, make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]));
      }
      // rescale the output row when the reference max moved (O is overwritten at t == 0)
      if (t > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        uint32_t o[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_o + lane_off + static_cast<uint32_t>(c * 32), o[c]);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[c][i] = __float_as_uint(__uint_as_float(o[c][i]) * alpha);
          tmem_st_32x32b_x32(t_o + lane_off + static_cast<uint32_t>(c * 32), o[c]);
        }
        tmem_st_wait();
      }
      fence_proxy_async_smem();  // P visible to the MMA (async proxy)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && warp_poll(pv_done, static_cast<uint32_t>((nt - 1) & 1), err, kDevErrTimeoutTmemFull, lane)) {
      tc_fence_after();
      const float inv_l = 1.0f / l;
      // out row -> the Q buffer (free: every S MMA has completed), as two 32 x 64
      // boxes per warp per 64-column half, then TMA stores
      const uint32_t stage = base + AttSmem::kQ + static_cast<uint32_t>(quad * 2 * 32 * 128);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(t_o + lane_off + static_cast<uint32_t>(c * 32), o);
        tmem_ld_wait();
        const uint32_t box = stage + static_cast<uint32_t>((c >> 1) * 32 * 128);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = (c & 1) * 4 + q;
          const uint4 w = make_uint4(pack_bf16x2(__uint_as_float(o[8 * q]) * inv_l, __uint_as_float(o[8 * q + 1]) * inv_l),
                                     pack_bf16x2(__uint_as_float(o[8 * q + 2]) * inv_l, __uint_as_float(o[8 * q + 3]) * inv_l),
                                     pack_bf16x2(__uint_as_float(o[8 * q + 4]) * inv_l, __uint_as_float(o[8 * q + 5]) * inv_l),
                                     pack_bf16x2(__uint_as_float(o[8 * q + 6]) * inv_l, __uint_as_float(o[8 * q + 7]) * inv_l));
          st_shared_v4(box + static_cast<uint32_t>(lane * 128 + ((ch ^ (lane & 7)) << 4)), w);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmO, h * kAttD, row_q + quad * 32, stage);
        tma_store_2d(&tmO, h * kAttD + 64, row_q + quad * 32, stage + 32 * 128);
        bulk_commit_group();
      }
      if (qpos < p.T)
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
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse = lse;
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  const int smem = AttSmem::kBytes + 1024;
  static_assert(AttSmem::kBytes + 1024 <= 232448, "shared memory budget exceeded");
  if (cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HLM_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t grid = B * H * (T / kAttBQ);
  {
    LaunchScope scope(HLM_KERNEL_ATTN_FWD, s);
    attn_fwd_kernel<<<static_cast<unsigned>(grid), 192, smem, s>>>(mq, mk, mv, mo, p);
  }
  return launch_status();
}
