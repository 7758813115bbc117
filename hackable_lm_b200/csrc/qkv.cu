// Fused QKV projection + QK-norm + RoPE (forward) and its backward.
//
// Forward = one tcgen05 GEMM  qkv = X @ W_qkv^T  with BN = 256, so each
// output tile is exactly two heads of 128 token rows.  The epilogue owns
// whole head rows (one row per thread): for q/k heads it computes the RMS
// over the 128 fp32 accumulators, normalises, rotates the first rotary_dim
// dims (rotate-half, cos/sin[t, d mod half]) and writes [B,T,H,D] through TMA
// stores; v heads are written as they are.  This replaces the reference's GEMM -> bf16 qkv ->
// strided split -> qk_norm_rope chain (model.py:92-99, 117-126;
// kernels.py:446-503) with one pass over the output.
//
// Backward: a memory-bound kernel (qk_norm_rope.cu, mode kRopeBwdY) recovers
// the normalised vectors from the saved outputs (inverse rotation) and the
// saved 1/rms, applies the norm/RoPE backward (kernels.py:546-612) to produce
// dq_pre/dk_pre, then two
// tcgen05 GEMMs read [dq_pre | dk_pre | dv] as one segmented operand:
//   grad_x = [dq|dk|dv] @ W_qkv          (W read N-major)
//   grad_w = [dq|dk|dv]^T @ X            (split-K; the splits add their fp32 partials
//                                         into one buffer in L2, which one pass rounds to
//                                         bf16; the fp32 sum order varies run to run)
#include "gemm_sm100.cuh"
#include "rope_vec.cuh"

namespace hlm {

constexpr int kQkvD = 128;
constexpr int kQkvBN = 2 * kQkvD;  // two heads per output tile
constexpr int kQkvStages = 6;     // CTA-pair stages: 16 KB of A + 16 KB (half) of B
constexpr int kQkvEpiWarps = 4;  // 8 (one warp per lane quadrant and head) spills registers
constexpr int kDwBN = 256;

// Forward epilogue: the tile holds 128 token rows x 2 heads (BN = 256).  Each
// thread owns one row.  Per head: 4 x tcgen05.ld (128 fp32), then for q/k
// heads RMSNorm over the 128 values + rotate-half RoPE on the first RD dims
// (cos/sin of the row's position loaded once per tile), v heads pass through;
// the bf16 row is staged in 128B-swizzled shared memory (two 32x64 boxes per
// warp) and written with TMA tensor stores (full 128-byte lines).
template <int RD>
struct EpiQKV {
  struct Params {
    alignas(64) CUtensorMap map_q;  // q_out as [M][Hq*128] bf16, box {64, 32}
    alignas(64) CUtensorMap map_k;  // k_out as [M][Hk*128]
    alignas(64) CUtensorMap map_v;  // v_out as [M][Hk*128]
    float* rstd;
    const void* cosp;
    const void* sinp;
    int64_t cs_stride;
    int cs_dtype;
    int T, Hq, Hk;
    float eps;
  };
  static constexpr int kBoxBytes = 32 * 128;
  // per epilogue warp: one head = 2 boxes
  template <int EPI_WARPS>
  static constexpr int smem_bytes() {
    return EPI_WARPS * 2 * kBoxBytes;
  }

  // With two warps per lane quadrant (kParts = 2) warp `part` takes head
  // `part` of the tile; with one it takes both in turn.
  template <int BN, int kParts>
  static HLM_DEVICE void run(const Params& ep, const GemmParams& p, uint8_t* smem, uint32_t taddr,
                             int m_tile, int n_tile, int, int quad, int part, int lane) {
    static_assert(BN == 2 * kQkvD, "two heads per tile");
    static_assert(kParts == 1 || kParts == 2, "one or two warps per lane quadrant");
    const int row = m_tile * kBM + quad * 32 + lane;
    const bool row_ok = row < p.M;
    const int Hq = ep.Hq, Hk = ep.Hk, nqk = Hq + Hk, nh = Hq + 2 * Hk;
    const float eps = ep.eps;
    float* const rstd = ep.rstd;
    const uint32_t buf =
        smem_u32(smem) + static_cast<uint32_t>((part * 4 + quad) * 2 * kBoxBytes);
    // cos/sin of this row's position, first RD/2 entries (shared by both heads)
    float cv[RD > 0 ? RD / 2 : 1], sv[RD > 0 ? RD / 2 : 1];
    if constexpr (RD > 0) {
      const int64_t t = row_ok ? row % ep.T : 0;
      if (ep.cs_dtype == HLM_F32) {
        const float* cp = static_cast<const float*>(ep.cosp) + t * ep.cs_stride;
        const float* sp = static_cast<const float*>(ep.sinp) + t * ep.cs_stride;
#pragma unroll
        for (int i = 0; i < RD / 2; i += 4) {
          const float4 c4 = *reinterpret_cast<const float4*>(cp + i);
          const float4 s4 = *reinterpret_cast<const float4*>(sp + i);
          cv[i] = c4.x; cv[i + 1] = c4.y; cv[i + 2] = c4.z; cv[i + 3] = c4.w;
          sv[i] = s4.x; sv[i + 1] = s4.y; sv[i + 2] = s4.z; sv[i + 3] = s4.w;
        }
      } else {
        const __nv_bfloat16* cp = static_cast<const __nv_bfloat16*>(ep.cosp) + t * ep.cs_stride;
        const __nv_bfloat16* sp = static_cast<const __nv_bfloat16*>(ep.sinp) + t * ep.cs_stride;
#pragma unroll
        for (int i = 0; i < RD / 2; i += 8) {
          Vec16<__nv_bfloat16> c8, s8;
          c8.raw = ld_global_nc_v4(cp + i);
          s8.raw = ld_global_nc_v4(sp + i);
          float cf[8], sf[8];
          c8.to_float(cf);
          s8.to_float(sf);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            cv[i + j] = cf[j];
            sv[i + j] = sf[j];
          }
        }
      }
    }
#pragma unroll 1
    for (int hs = kParts == 2 ? part : 0; hs < 2; hs += kParts) {
      const int head = n_tile * 2 + hs;
      uint32_t r0[32], r1[32], r2[32], r3[32];
      const uint32_t ta = taddr + static_cast<uint32_t>(hs * kQkvD);
      tmem_ld_32x32b_x32(ta + 0u, r0);
      tmem_ld_32x32b_x32(ta + 32u, r1);
      tmem_ld_32x32b_x32(ta + 64u, r2);
      tmem_ld_32x32b_x32(ta + 96u, r3);
      tmem_ld_wait();
      if (head >= nh) continue;  // past the last head (odd head count): nothing to store
      float v[kQkvD];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        v[i] = __uint_as_float(r0[i]);
        v[32 + i] = __uint_as_float(r1[i]);
        v[64 + i] = __uint_as_float(r2[i]);
        v[96 + i] = __uint_as_float(r3[i]);
      }
      if (head < nqk) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < kQkvD; ++i) ss = fmaf(v[i], v[i], ss);
        const float inv = rsqrtf(ss * (1.0f / kQkvD) + eps);
#pragma unroll
        for (int i = 0; i < kQkvD; ++i) v[i] *= inv;
        if constexpr (RD > 0) {
#pragma unroll
          for (int i = 0; i < RD / 2; ++i) {
            const float a = v[i], b = v[i + RD / 2];
            v[i] = a * cv[i] - b * sv[i];
            v[i + RD / 2] = b * cv[i] + a * sv[i];
          }
        }
        if (row_ok) rstd[static_cast<int64_t>(row) * nqk + head] = inv;
      }
      // stage the bf16 row as two 32x64 boxes (128B swizzle) and store with TMA
      if (kParts == 1 && hs > 0) {
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
      }
#pragma unroll
      for (int b = 0; b < 2; ++b) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int e = b * 64 + c * 8;
          uint32_t w[4];
#pragma unroll
          for (int k2 = 0; k2 < 4; ++k2) {
            const __nv_bfloat162 h2 = __floats2bfloat162_rn(v[e + 2 * k2], v[e + 2 * k2 + 1]);
            w[k2] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          st_shared_v4(buf + static_cast<uint32_t>(b * kBoxBytes + lane * 128 + ((c ^ (lane & 7)) << 4)),
                       make_uint4(w[0], w[1], w[2], w[3]));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const CUtensorMap* map = head < Hq ? &ep.map_q : (head < nqk ? &ep.map_k : &ep.map_v);
        const int hh = head < Hq ? head : (head < nqk ? head - Hq : head - nqk);
        const int r0w = m_tile * kBM + quad * 32;
        tma_store_2d(map, hh * kQkvD, r0w, buf);
        tma_store_2d(map, hh * kQkvD + 64, r0w, buf + kBoxBytes);
        bulk_commit_group();
      }
    }
    if (lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
  }
};

__global__ void __launch_bounds__(256) splitk_reduce_bf16_kernel(const float* __restrict__ slabs,
                                                                int splits, int64_t n,
                                                                __nv_bfloat16* __restrict__ out) {
  const int64_t nv = n / 4;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < nv;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 acc = reinterpret_cast<const float4*>(slabs)[v];
    for (int sidx = 1; sidx < splits; ++sidx) {
      const float4 x = reinterpret_cast<const float4*>(slabs + static_cast<int64_t>(sidx) * n)[v];
      acc.x += x.x;
      acc.y += x.y;
      acc.z += x.z;
      acc.w += x.w;
    }
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(out + v * 4);
    o[0] = __floats2bfloat162_rn(acc.x, acc.y);
    o[1] = __floats2bfloat162_rn(acc.z, acc.w);
  }
}

// Split-K count for the dW GEMM (few output tiles, long K): the smallest split
// whose work units (256 x kDwBN pair tiles) fill the CTA-pair waves to >= 95%
// (the splits add their fp32 partials into one L2-resident buffer, so a split
// costs its reductions, not a slab), else the best fill found up to 16 splits;
// every split keeps at least 8 K blocks.
static inline int qkv_dw_splits(int64_t tokens, int64_t nqkv, int64_t C) {
  const int64_t tiles = ((nqkv + 2 * kBM - 1) / (2 * kBM)) * ((C + kDwBN - 1) / kDwBN);
  const int64_t kblocks = (tokens + kBK - 1) / kBK;
  const int64_t sms = num_sms_of_current_device() / 2;  // CTA pairs
  int best = 1;
  double best_fill = 0.0;
  for (int64_t s = 1; s <= 16 && s <= kblocks / 8; ++s) {
    // gemm_tiling may merge splits; evaluate the effective count
    const int64_t kb_per = (kblocks + s - 1) / s;
    const int64_t eff = (kblocks + kb_per - 1) / kb_per;
    const int64_t units = tiles * eff;
    const double fill = static_cast<double>(units) / (((units + sms - 1) / sms) * sms);
    if (fill > best_fill + 1e-9) {
      best_fill = fill;
      best = static_cast<int>(eff);
    }
    if (fill >= 0.95) break;
  }
  return best;
}

static inline size_t a256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

struct QkvBwdPlan {
  int splits;
  size_t off_dq, off_dk, off_slab, total;
};

static QkvBwdPlan qkv_bwd_plan(int64_t M, int64_t C, int64_t Hq, int64_t Hk) {
  QkvBwdPlan pl;
  const int64_t nqkv = (Hq + 2 * Hk) * kQkvD;
  pl.splits = qkv_dw_splits(M, nqkv, C);
  size_t off = 0;
  pl.off_dq = off;
  off = a256(off + static_cast<size_t>(M) * Hq * kQkvD * 2);
  pl.off_dk = off;
  off = a256(off + static_cast<size_t>(M) * Hk * kQkvD * 2);
  pl.off_slab = off;  // fp32 dW accumulated by every split
  off = a256(off + static_cast<size_t>(nqkv) * C * 4);
  pl.total = off;
  return pl;
}

template <int RD>
static int qkv_fwd_launch(const CUtensorMap& mx, const CUtensorMap& mw, const GemmParams& p,
                          const typename EpiQKV<RD>::Params& ep, cudaStream_t s) {
  return launch_gemm_pair<kQkvBN, kQkvStages, false, false, EpiQKV<RD>, kQkvEpiWarps>(
      mx, mx, mx, mw, p, ep, s, HLM_KERNEL_QKV_FWD);
}

}  // namespace hlm

using namespace hlm;

extern "C" int hlm_qkv_rope_fwd(const void* x, const void* w_qkv, const void* cos, const void* sin,
                                void* q_out, void* k_out, void* v_out, float* rstd, int64_t B,
                                int64_t T, int64_t C, int64_t Hq, int64_t Hk, int64_t D,
                                int64_t rotary_dim, int64_t cs_stride_t, int cs_dtype, float eps,
                                void* stream) {
  if (B < 0 || T <= 0 || C <= 0 || Hq <= 0 || Hk <= 0 || D <= 0) return HLM_ERR_INVALID_ARG;
  if (D != kQkvD) return HLM_ERR_UNSUPPORTED;
  const int64_t M = B * T;
  if (M == 0) return HLM_OK;
  if (x == nullptr || w_qkv == nullptr || q_out == nullptr || k_out == nullptr ||
      v_out == nullptr || rstd == nullptr)
    return HLM_ERR_INVALID_ARG;
  if (rotary_dim > 0 && (cos == nullptr || sin == nullptr)) return HLM_ERR_INVALID_ARG;
  if (C % 64 != 0 || M > (1ll << 31) - 256) return HLM_ERR_UNSUPPORTED;
  if (cs_dtype != HLM_F32 && cs_dtype != HLM_BF16 && cs_dtype != HLM_F16) return HLM_ERR_UNSUPPORTED;
  if (!host_aligned16(x) || !host_aligned16(w_qkv) || !host_aligned16(q_out) ||
      !host_aligned16(k_out) || !host_aligned16(v_out))
    return HLM_ERR_UNSUPPORTED;
  const int64_t nqkv = (Hq + 2 * Hk) * kQkvD;
  CUtensorMap mx, mw;
  if (!encode_bf16_map(&mx, x, C, M, C, kBM)) return HLM_ERR_DRIVER;
  if (!encode_bf16_map(&mw, w_qkv, C, nqkv, C, 64)) return HLM_ERR_DRIVER;  // pair: 64-row boxes of B
  if (rotary_dim > 0 && (!host_aligned16(cos) || !host_aligned16(sin) ||
                         (cs_stride_t * (cs_dtype == HLM_F32 ? 4 : 2)) % 16 != 0))
    return HLM_ERR_UNSUPPORTED;
  if (cs_dtype == HLM_F16) return HLM_ERR_UNSUPPORTED;
  GemmParams p;
  gemm_tiling_pair(p, static_cast<int>(M), static_cast<int>(nqkv), static_cast<int>(C), kQkvBN, 1);
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define HLM_QKV_CASE(RDV)                                  \
  case RDV: {                                              \
    EpiQKV<RDV>::Params ep;                                \
    if (!encode_bf16_map(&ep.map_q, q_out, Hq * kQkvD, M, Hq * kQkvD, 32) ||   \
        !encode_bf16_map(&ep.map_k, k_out, Hk * kQkvD, M, Hk * kQkvD, 32) ||   \
        !encode_bf16_map(&ep.map_v, v_out, Hk * kQkvD, M, Hk * kQkvD, 32))     \
      return HLM_ERR_DRIVER;                               \
    ep.rstd = rstd;                                        \
    ep.cosp = cos;                                         \
    ep.sinp = sin;                                         \
    ep.cs_stride = cs_stride_t;                            \
    ep.cs_dtype = cs_dtype;                                \
    ep.T = static_cast<int>(T);                            \
    ep.Hq = static_cast<int>(Hq);                          \
    ep.Hk = static_cast<int>(Hk);                          \
    ep.eps = eps;                                          \
    return qkv_fwd_launch<RDV>(mx, mw, p, ep, s);          \
  }
  switch (rotary_dim) {
    HLM_QKV_CASE(0)
    HLM_QKV_CASE(16)
    HLM_QKV_CASE(32)
    HLM_QKV_CASE(64)
    HLM_QKV_CASE(128)
    default:
      return HLM_ERR_UNSUPPORTED;
  }
#undef HLM_QKV_CASE
}

extern "C" size_t hlm_qkv_rope_bwd_workspace_bytes(int64_t B, int64_t T, int64_t C, int64_t Hq,
                                                   int64_t Hk, int64_t D) {
  (void)D;
  if (B <= 0 || T <= 0 || C <= 0 || Hq <= 0 || Hk <= 0) return 256;
  return qkv_bwd_plan(B * T, C, Hq, Hk).total;
}

extern "C" int hlm_qkv_rope_bwd(const void* x, const void* w_qkv, const void* q_out,
                                const void* k_out, const float* rstd, const void* cos,
                                const void* sin, const void* grad_q, const void* grad_k,
                                const void* grad_v, void* grad_x, void* grad_w, void* workspace,
                                size_t workspace_bytes, int64_t B, int64_t T, int64_t C,
                                int64_t Hq, int64_t Hk, int64_t D, int64_t rotary_dim,
                                int64_t cs_stride_t, int cs_dtype, float eps, void* stream) {
  if (B < 0 || T <= 0 || C <= 0 || Hq <= 0 || Hk <= 0 || D <= 0) return HLM_ERR_INVALID_ARG;
  if (D != kQkvD) return HLM_ERR_UNSUPPORTED;
  if (rotary_dim < 0 || rotary_dim > D || (rotary_dim / 2) % 8 != 0 || (rotary_dim & 1))
    return HLM_ERR_UNSUPPORTED;
  const int64_t M = B * T;
  if (M == 0) return HLM_OK;
  if (x == nullptr || w_qkv == nullptr || q_out == nullptr || k_out == nullptr ||
      rstd == nullptr || grad_q == nullptr || grad_k == nullptr || grad_v == nullptr ||
      workspace == nullptr)
    return HLM_ERR_INVALID_ARG;
  if (rotary_dim > 0 && (cos == nullptr || sin == nullptr)) return HLM_ERR_INVALID_ARG;
  if (C % 64 != 0 || M > (1ll << 31) - 256) return HLM_ERR_UNSUPPORTED;
  if (cs_dtype != HLM_F32 && cs_dtype != HLM_BF16) return HLM_ERR_UNSUPPORTED;
  if (rotary_dim > 0 && (!host_aligned16(cos) || !host_aligned16(sin) ||
                         (cs_stride_t * (cs_dtype == HLM_F32 ? 4 : 2)) % 16 != 0))
    return HLM_ERR_UNSUPPORTED;
  if (B * T * (Hq + Hk) >= (1ll << 31)) return HLM_ERR_UNSUPPORTED;
  const void* ptrs[] = {x, w_qkv, q_out, k_out, grad_q, grad_k, grad_v, workspace};
  for (const void* ptr : ptrs)
    if (!host_aligned16(ptr)) return HLM_ERR_UNSUPPORTED;
  if ((grad_x != nullptr && !host_aligned16(grad_x)) || (grad_w != nullptr && !host_aligned16(grad_w)))
    return HLM_ERR_UNSUPPORTED;
  const QkvBwdPlan pl = qkv_bwd_plan(M, C, Hq, Hk);
  if (workspace_bytes < pl.total) return HLM_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* dq = reinterpret_cast<__nv_bfloat16*>(ws + pl.off_dq);
  __nv_bfloat16* dk = reinterpret_cast<__nv_bfloat16*>(ws + pl.off_dk);
  float* slabs = reinterpret_cast<float*>(ws + pl.off_slab);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = device_error_ptr();
  if (err == nullptr) return HLM_ERR_LAUNCH;
  const int64_t nqkv = (Hq + 2 * Hk) * kQkvD;

  // 1. norm + RoPE backward -> dq_pre, dk_pre, from the saved outputs and 1/rms
  {
    RopeArgs a{};
    a.xq = q_out;
    a.xk = k_out;
    a.gq = grad_q;
    a.gk = grad_k;
    a.rstd = rstd;
    a.cosp = cos;
    a.sinp = sin;
    a.oq = dq;
    a.ok = dk;
    a.qs0 = T * Hq * kQkvD;
    a.qs1 = Hq * kQkvD;
    a.qs2 = kQkvD;
    a.ks0 = T * Hk * kQkvD;
    a.ks1 = Hk * kQkvD;
    a.ks2 = kQkvD;
    a.cs_stride = cs_stride_t;
    a.tokens = static_cast<uint32_t>(M);
    a.T = static_cast<uint32_t>(T);
    a.Hq = static_cast<int>(Hq);
    a.Hk = static_cast<int>(Hk);
    a.D = kQkvD;
    a.rd = static_cast<int>(rotary_dim);
    a.eps = eps;
    const int rc = rope_vec_launch<__nv_bfloat16, kRopeBwdY>(a, cs_dtype, HLM_KERNEL_QKV_BWD_NORM, s);
    if (rc != HLM_OK) return rc;
  }
  const int seg1 = static_cast<int>(Hq * kQkvD);
  const int seg2 = static_cast<int>((Hq + Hk) * kQkvD);
  // grad_w (step 3) runs on the library's side stream, forked here and joined at the
  // end, so that its CTAs take the SMs grad_x's last wave leaves idle (the two GEMMs
  // are independent; each holds one CTA per SM)
  SideStream* side = nullptr;
  std::unique_lock<std::mutex> side_lock;
  cudaStream_t sw = s;
  if (grad_x != nullptr && grad_w != nullptr) {
    side = side_stream_of_current_device();
    if (side == nullptr) return HLM_ERR_LAUNCH;
    side_lock = std::unique_lock<std::mutex>(side->mu);
    if (cudaEventRecord(side->ev_start, s) != cudaSuccess ||
        cudaStreamWaitEvent(side->stream, side->ev_start, 0) != cudaSuccess)
      return HLM_ERR_LAUNCH;
    sw = side->stream;
  }
  // 2. grad_x = [dq|dk|dv] @ W_qkv
  if (grad_x != nullptr) {
    CUtensorMap a0, a1, a2, mb;
    if (!encode_bf16_map(&a0, dq, Hq * kQkvD, M, Hq * kQkvD, kBM) ||
        !encode_bf16_map(&a1, dk, Hk * kQkvD, M, Hk * kQkvD, kBM) ||
        !encode_bf16_map(&a2, grad_v, Hk * kQkvD, M, Hk * kQkvD, kBM) ||
        !encode_bf16_map(&mb, w_qkv, C, nqkv, C, 64))
      return HLM_ERR_DRIVER;
    GemmParams p;
    gemm_tiling_pair(p, static_cast<int>(M), static_cast<int>(C), static_cast<int>(nqkv), kDwBN, 1);
    p.a_seg1 = seg1;
    p.a_seg2 = seg2;
    p.err = err;
    EpiStore::Params ep;
    ep.d = grad_x;
    ep.ldd = C;
    ep.split_stride = 0;
    ep.dtype = HLM_BF16;
    ep.accumulate = 0;
    ep.vec_ok = 1;
    ep.alpha = nullptr;
    const int rc = launch_gemm_pair<kDwBN, kQkvStages, false, true, EpiStore>(a0, a1, a2, mb, p, ep, s,
                                                                             HLM_KERNEL_QKV_DX);
    if (rc != HLM_OK) return rc;
  }
  // 3. grad_w = [dq|dk|dv]^T @ X   (split-K over tokens)
  if (grad_w != nullptr) {
    CUtensorMap a0, a1, a2, mb;
    if (!encode_bf16_map(&a0, dq, Hq * kQkvD, M, Hq * kQkvD, 64) ||
        !encode_bf16_map(&a1, dk, Hk * kQkvD, M, Hk * kQkvD, 64) ||
        !encode_bf16_map(&a2, grad_v, Hk * kQkvD, M, Hk * kQkvD, 64) ||
        !encode_bf16_map(&mb, x, C, M, C, 64))
      return HLM_ERR_DRIVER;
    GemmParams p;
    gemm_tiling_pair(p, static_cast<int>(nqkv), static_cast<int>(C), static_cast<int>(M), kDwBN,
                     pl.splits);
    if (p.splits != pl.splits) return HLM_ERR_LAUNCH;
    p.a_seg1 = seg1;
    p.a_seg2 = seg2;
    p.err = err;
    // the splits add into one fp32 dW (zeroed first), then one pass rounds it to bf16
    const int64_t n = nqkv * C;
    if (cudaMemsetAsync(slabs, 0, static_cast<size_t>(n) * sizeof(float), sw) != cudaSuccess)
      return HLM_ERR_LAUNCH;
    EpiStore::Params ep;
    ep.d = slabs;
    ep.ldd = C;
    ep.split_stride = 0;
    ep.dtype = HLM_F32;
    ep.accumulate = 2;
    ep.vec_ok = 1;
    ep.alpha = nullptr;
    const int rc = launch_gemm_pair<kDwBN, kQkvStages, true, true, EpiStore>(a0, a1, a2, mb, p, ep, sw,
                                                                            HLM_KERNEL_QKV_DW);
    if (rc != HLM_OK) return rc;
    int64_t blocks = (n / 4 + 255) / 256;
    const int64_t cap = static_cast<int64_t>(num_sms_of_current_device()) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    {
      LaunchScope scope(0, sw);
      splitk_reduce_bf16_kernel<<<static_cast<int>(blocks), 256, 0, sw>>>(
          slabs, 1, n, static_cast<__nv_bfloat16*>(grad_w));
    }
    if (launch_status() != HLM_OK) return HLM_ERR_LAUNCH;
  }
  if (side != nullptr && (cudaEventRecord(side->ev_done[0], side->stream) != cudaSuccess ||
                          cudaStreamWaitEvent(s, side->ev_done[0], 0) != cudaSuccess))
    return HLM_ERR_LAUNCH;
  return HLM_OK;
}
