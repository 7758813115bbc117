// QK-norm + partial rotate-half RoPE, forward and backward, on strided q/k
// views (the packed qkv GEMM output viewed as [B,T,H,D] with row stride
// (Hq+2Hk)*D).  Semantics follow kernels.py:446-503 (forward) and
// kernels.py:546-612 (backward):
//   forward : z = x*rsqrt(mean(x^2)+eps); rotate the first rotary_dim dims of
//             z with cos/sin[t, d mod half]; pass-through dims are z.
//   backward: g_n = inverse rotation of g; dx = inv*(g_n - z*mean(g_n*z)).
//
// Vector path: one head vector is spread over LPH = D/VEC lanes, each lane
// holding one 16-byte vector; a warp walks the heads of one token at a time.
// The rotation partner of a lane's vector is re-read (an L1 hit); the sum of
// squares and the backward dot product are shuffle-xor reductions inside the
// LPH-lane group.
#include <type_traits>

#include "rope_vec.cuh"

namespace hlm {

struct QKShape {
  int64_t B, T, Hq, Hk, D, rd;
  int64_t qs[4], ks[4];
  int64_t cs_stride;
  int cs_dtype;
  float eps;
};

template <int LPH>
HLM_DEVICE float group_sum(float v) {
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// VEC consecutive cos/sin entries as fp32 (16-byte vector loads; the host
// checks alignment before choosing this path).
template <typename CS, int VEC>
HLM_DEVICE void load_cs_vec(const CS* p, float (&out)[VEC]) {
  constexpr int PER = 16 / sizeof(CS);
#pragma unroll
  for (int v = 0; v < VEC / PER; ++v) {
    Vec16<CS> raw;
    raw.raw = ld_global_v4(p + v * PER);
    float f[PER];
    raw.to_float(f);
#pragma unroll
    for (int i = 0; i < PER; ++i) out[v * PER + i] = f[i];
  }
}

// Token-major vector kernel: a warp owns one token at a time and walks its
// H = Hq + Hk head vectors HPW = 32/LPH at a time (one LPH-lane group per
// head vector, lane = VEC consecutive dims).  Everything that depends only on
// the token and the lane -- the batch/position index math and the lane's
// cos/sin slice with its rotation role folded in -- is computed once per token
// and reused for every head.  U passes of loads are issued before any of them
// is used (the lane's 16 bytes, its rotation partner's 16 bytes -- a re-read
// that hits L1, cheaper than shuffles -- and for the backward the gradient
// pair), then the rotation is branch-free:
//   out = inv * (x*c' + sgn*s*px),  c' = cos (rotated dims) or 1 (pass-through),
//   sgn = -1 for d < rd/2, +1 for rd/2 <= d < rd, 0 beyond.
// Modes: kRopeFwd (x -> rotated norm), kRopeBwdX (x, g -> dx),
//        kRopeBwdY (saved output y, saved 1/rms, g -> dx; the normalised
//        vector z is the inverse rotation of y).
template <typename T, typename CS, int LPH, int MODE, int U>
__global__ void __launch_bounds__(256) qk_norm_rope_vec_kernel(const RopeArgs a) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int HPW = 32 / LPH;
  const int lane = threadIdx.x & 31;
  const int slot = lane / LPH, li = lane % LPH;
  const int H = a.Hq + a.Hk;
  const int Hq = a.Hq;
  const int D = a.D;
  const int half = a.rd / 2, d0 = li * VEC;
  const int role = d0 < half ? 0 : (d0 < a.rd ? 1 : 2);
  const int pdim = role == 0 ? d0 + half : (role == 1 ? d0 - half : d0);
  const int cb = role == 2 ? 0 : (role == 0 ? d0 : d0 - half);
  const float sgn = role == 0 ? -1.0f : (role == 1 ? 1.0f : 0.0f);
  const float cpass = role == 2 ? 1.0f : 0.0f;  // c' = cpass + crot * cos
  const float crot = 1.0f - cpass;
  const bool has_rot = a.rd > 0;
  const float inv_d = 1.0f / static_cast<float>(D);
  const T* xq = static_cast<const T*>(a.xq);
  const T* xk = static_cast<const T*>(a.xk);
  const int passes = (H + HPW - 1) / HPW;
  const uint32_t nwarps = gridDim.x * (blockDim.x >> 5);
  for (uint32_t tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); tok < a.tokens;
       tok += nwarps) {
    const uint32_t b = tok / a.T, t = tok - b * a.T;
    float c[VEC], s[VEC];
    if (has_rot) {
      load_cs_vec<CS, VEC>(static_cast<const CS*>(a.cosp) + t * a.cs_stride + cb, c);
      load_cs_vec<CS, VEC>(static_cast<const CS*>(a.sinp) + t * a.cs_stride + cb, s);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) c[i] = s[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      c[i] = fmaf(crot, c[i], cpass);
      s[i] *= sgn;
    }
    const T* qrow = xq + b * a.qs0 + t * a.qs1;
    const T* krow = xk + b * a.ks0 + t * a.ks1;
    const int64_t qo = static_cast<int64_t>(tok) * Hq * D;  // outputs / grads: contiguous
    const int64_t ko = static_cast<int64_t>(tok) * a.Hk * D;
    for (int p0 = 0; p0 < passes; p0 += U) {
      uint4 xr[U], pr[U], gr[U], pgr[U];
      float rs[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int h = (p0 + u) * HPW + slot;
        const int hc = h < H ? h : 0;
        const bool is_q = hc < Hq;
        const int hh = is_q ? hc : hc - Hq;
        const T* row = is_q ? qrow + hh * a.qs2 : krow + hh * a.ks2;
        xr[u] = ld_global_nc_l1_v4(row + d0);
        pr[u] = ld_global_nc_l1_v4(row + pdim);
        if constexpr (MODE != kRopeFwd) {
          const T* grow = static_cast<const T*>(is_q ? a.gq : a.gk) + (is_q ? qo : ko) +
                          static_cast<int64_t>(hh) * D;
          gr[u] = ld_global_nc_l1_v4(grow + d0);
          pgr[u] = ld_global_nc_l1_v4(grow + pdim);
        }
        if constexpr (MODE == kRopeBwdY) rs[u] = a.rstd[static_cast<int64_t>(tok) * H + hc];
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int h = (p0 + u) * HPW + slot;
        float x[VEC], px[VEC], res[VEC];
        {
          Vec16<T> v, pv;
          v.raw = xr[u];
          pv.raw = pr[u];
          v.to_float(x);
          pv.to_float(px);
        }
        if constexpr (MODE == kRopeFwd) {
          float ss = 0.0f;
#pragma unroll
          for (int i = 0; i < VEC; ++i) ss = fmaf(x[i], x[i], ss);
          ss = group_sum<LPH>(ss);
          const float inv = rsqrtf(ss * inv_d + a.eps);
#pragma unroll
          for (int i = 0; i < VEC; ++i) res[i] = inv * fmaf(s[i], px[i], x[i] * c[i]);
        } else {
          float g[VEC], pg[VEC];
          {
            Vec16<T> v, pv;
            v.raw = gr[u];
            pv.raw = pgr[u];
            v.to_float(g);
            pv.to_float(pg);
          }
          float inv, z[VEC];
          if constexpr (MODE == kRopeBwdX) {
            float ss = 0.0f;
#pragma unroll
            for (int i = 0; i < VEC; ++i) ss = fmaf(x[i], x[i], ss);
            ss = group_sum<LPH>(ss);
            inv = rsqrtf(ss * inv_d + a.eps);
#pragma unroll
            for (int i = 0; i < VEC; ++i) z[i] = x[i] * inv;
          } else {
            inv = rs[u];
            // inverse rotation of the saved output y gives the normalised vector
#pragma unroll
            for (int i = 0; i < VEC; ++i) z[i] = fmaf(-s[i], px[i], x[i] * c[i]);
          }
          // inverse rotation of the output gradient
          float dot = 0.0f, gn[VEC];
#pragma unroll
          for (int i = 0; i < VEC; ++i) {
            gn[i] = fmaf(-s[i], pg[i], g[i] * c[i]);
            dot = fmaf(gn[i], z[i], dot);
          }
          dot = group_sum<LPH>(dot) * inv_d;
#pragma unroll
          for (int i = 0; i < VEC; ++i) res[i] = inv * fmaf(-z[i], dot, gn[i]);
        }
        if (h < H) {
          const bool is_q = h < Hq;
          const int hh = is_q ? h : h - Hq;
          Vec16<T> o;
          o.from_float(res);
          st_global_v4(static_cast<T*>(is_q ? a.oq : a.ok) + (is_q ? qo : ko) +
                           static_cast<int64_t>(hh) * D + d0,
                       o.raw);
        }
      }
    }
  }
}

// Scalar path for any D / rotary_dim / stride: one warp per head vector, the
// rotation partner re-read from memory (as the reference Triton kernel does).
template <typename T, bool BWD>
__global__ void __launch_bounds__(256) qk_norm_rope_scalar_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ gq,
    const T* __restrict__ gk, const void* __restrict__ cosp, const void* __restrict__ sinp,
    T* __restrict__ q_out, T* __restrict__ k_out, QKShape sh) {
  const int lane = threadIdx.x & 31;
  const int64_t H = sh.Hq + sh.Hk;
  const int64_t total = sh.B * sh.T * H;
  const int64_t half = sh.rd / 2;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       item < total; item += warps_total) {
    const int64_t h = item % H;
    const int64_t bt = item / H;
    const int64_t t = bt % sh.T;
    const int64_t b = bt / sh.T;
    const bool is_q = h < sh.Hq;
    const int64_t hh = is_q ? h : h - sh.Hq;
    const int64_t* st = is_q ? sh.qs : sh.ks;
    const T* src = (is_q ? q : k) + b * st[0] + t * st[1] + hh * st[2];
    const int64_t Hsel = is_q ? sh.Hq : sh.Hk;
    const int64_t out_off = ((b * sh.T + t) * Hsel + hh) * sh.D;
    float ss = 0.0f;
    for (int64_t d = lane; d < sh.D; d += 32) {
      const float v = to_f32(src[d * st[3]]);
      ss += v * v;
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / static_cast<float>(sh.D) + sh.eps);
    if constexpr (!BWD) {
      T* dst = (is_q ? q_out : k_out) + out_off;
      for (int64_t d = lane; d < sh.D; d += 32) {
        const float z = to_f32(src[d * st[3]]) * inv;
        float r = z;
        if (d < sh.rd) {
          const int64_t pi = d < half ? d + half : d - half;
          const int64_t ci = d < half ? d : d - half;
          const float pz = to_f32(src[pi * st[3]]) * inv;
          const float c = load_cs(cosp, t * sh.cs_stride + ci, sh.cs_dtype);
          const float s = load_cs(sinp, t * sh.cs_stride + ci, sh.cs_dtype);
          r = d < half ? z * c - pz * s : z * c + pz * s;
        }
        dst[d] = from_f32<T>(r);
      }
    } else {
      const T* g = (is_q ? gq : gk) + out_off;
      float dot = 0.0f;
      for (int64_t d = lane; d < sh.D; d += 32) {
        float gn = to_f32(g[d]);
        if (d < sh.rd) {
          const int64_t pi = d < half ? d + half : d - half;
          const int64_t ci = d < half ? d : d - half;
          const float c = load_cs(cosp, t * sh.cs_stride + ci, sh.cs_dtype);
          const float s = load_cs(sinp, t * sh.cs_stride + ci, sh.cs_dtype);
          const float pg = to_f32(g[pi]);
          gn = d < half ? gn * c + pg * s : gn * c - pg * s;
        }
        dot += gn * to_f32(src[d * st[3]]) * inv;
      }
      dot = warp_sum(dot) / static_cast<float>(sh.D);
      T* dst = (is_q ? q_out : k_out) + out_off;
      for (int64_t d = lane; d < sh.D; d += 32) {
        float gn = to_f32(g[d]);
        if (d < sh.rd) {
          const int64_t pi = d < half ? d + half : d - half;
          const int64_t ci = d < half ? d : d - half;
          const float c = load_cs(cosp, t * sh.cs_stride + ci, sh.cs_dtype);
          const float s = load_cs(sinp, t * sh.cs_stride + ci, sh.cs_dtype);
          const float pg = to_f32(g[pi]);
          gn = d < half ? gn * c + pg * s : gn * c - pg * s;
        }
        const float z = to_f32(src[d * st[3]]) * inv;
        dst[d] = from_f32<T>(inv * (gn - z * dot));
      }
    }
  }
}

// Loads in flight per lane: U passes of 2 (forward) or 4 (backward) vectors
// (measured: the backward's extra registers cost more than deeper batching gains).
template <int MODE>
constexpr int rope_passes_per_batch() {
  return MODE == kRopeFwd ? 3 : 1;
}

template <typename T, typename CS, int LPH, int MODE>
static void launch_rope_vec_lph(const RopeArgs& a, int64_t warps_needed, cudaStream_t s) {
  constexpr int U = rope_passes_per_batch<MODE>();
  auto kern = qk_norm_rope_vec_kernel<T, CS, LPH, MODE, U>;
  // persistent grid: as many 256-thread blocks as are resident at once
  static int per_sm = 0;
  if (per_sm == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 256, 0) != cudaSuccess || n < 1) n = 1;
    per_sm = n;
  }
  int64_t blocks = (warps_needed + 7) / 8;
  const int64_t cap = static_cast<int64_t>(num_sms_of_current_device()) * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  kern<<<static_cast<int>(blocks), 256, 0, s>>>(a);
}

template <typename T, typename CS, int MODE>
static void launch_rope_vec(int lph, const RopeArgs& a, int64_t warps_needed, cudaStream_t s) {
  switch (lph) {
    case 8:
      launch_rope_vec_lph<T, CS, 8, MODE>(a, warps_needed, s);
      break;
    case 16:
      launch_rope_vec_lph<T, CS, 16, MODE>(a, warps_needed, s);
      break;
    default:
      launch_rope_vec_lph<T, CS, 32, MODE>(a, warps_needed, s);
      break;
  }
}

// Vector-path launch shared by the standalone op and the fused QKV backward.
// Returns HLM_ERR_UNSUPPORTED when the layout does not allow 16-byte vectors.
template <typename T, int MODE>
int rope_vec_launch(const RopeArgs& a, int cs_dtype, int kernel_id, cudaStream_t s) {
  constexpr int VEC = 16 / sizeof(T);
  const int lph = a.D / VEC;
  bool vec = a.D % VEC == 0 && (lph == 8 || lph == 16 || lph == 32);
  vec = vec && (a.rd / 2) % VEC == 0 && a.rd <= a.D;
  const int64_t strides[] = {a.qs0, a.qs1, a.qs2, a.ks0, a.ks1, a.ks2};
  for (int64_t st : strides) vec = vec && st % VEC == 0;
  vec = vec && host_aligned16(a.xq) && host_aligned16(a.xk) && host_aligned16(a.oq) &&
        host_aligned16(a.ok);
  if (MODE != kRopeFwd) vec = vec && host_aligned16(a.gq) && host_aligned16(a.gk);
  const bool cs_same = (cs_dtype == HLM_F32 && sizeof(T) == 4) ||
                       (cs_dtype == HLM_BF16 && std::is_same<T, __nv_bfloat16>::value) ||
                       (cs_dtype == HLM_F16 && std::is_same<T, __half>::value);
  const bool cs_f32 = cs_dtype == HLM_F32;
  vec = vec && (cs_same || cs_f32);
  vec = vec && static_cast<int64_t>(a.tokens) * (a.Hq + a.Hk) < (1ll << 31);
  if (a.rd > 0)
    vec = vec && host_aligned16(a.cosp) && host_aligned16(a.sinp) &&
          (a.cs_stride * (cs_f32 ? 4 : 2)) % 16 == 0;
  if (!vec) return HLM_ERR_UNSUPPORTED;
  const int64_t warps = static_cast<int64_t>(a.tokens);  // one warp per token at a time
  LaunchScope scope(kernel_id, s);
  if (cs_f32)
    launch_rope_vec<T, float, MODE>(lph, a, warps, s);
  else
    launch_rope_vec<T, T, MODE>(lph, a, warps, s);
  return launch_status();
}

template int rope_vec_launch<__nv_bfloat16, kRopeBwdY>(const RopeArgs&, int, int, cudaStream_t);

template <typename T, bool BWD>
static int launch_qk_norm_rope(const void* q, const void* k, const void* gq, const void* gk,
                               const void* cosp, const void* sinp, void* q_out, void* k_out,
                               const QKShape& sh, cudaStream_t s) {
  if (sh.qs[3] == 1 && sh.ks[3] == 1 && sh.B * sh.T < (1ll << 31) && sh.T < (1ll << 31)) {
    RopeArgs a{};
    a.xq = q;
    a.xk = k;
    a.gq = gq;
    a.gk = gk;
    a.rstd = nullptr;
    a.cosp = cosp;
    a.sinp = sinp;
    a.oq = q_out;
    a.ok = k_out;
    a.qs0 = sh.qs[0];
    a.qs1 = sh.qs[1];
    a.qs2 = sh.qs[2];
    a.ks0 = sh.ks[0];
    a.ks1 = sh.ks[1];
    a.ks2 = sh.ks[2];
    a.cs_stride = sh.cs_stride;
    a.tokens = static_cast<uint32_t>(sh.B * sh.T);
    a.T = static_cast<uint32_t>(sh.T);
    a.Hq = static_cast<int>(sh.Hq);
    a.Hk = static_cast<int>(sh.Hk);
    a.D = static_cast<int>(sh.D);
    a.rd = static_cast<int>(sh.rd);
    a.eps = sh.eps;
    const int rc = BWD ? rope_vec_launch<T, kRopeBwdX>(a, sh.cs_dtype, HLM_KERNEL_QK_ROPE_BWD, s)
                       : rope_vec_launch<T, kRopeFwd>(a, sh.cs_dtype, HLM_KERNEL_QK_ROPE_FWD, s);
    if (rc != HLM_ERR_UNSUPPORTED) return rc;
  }
  const int64_t total = sh.B * sh.T * (sh.Hq + sh.Hk);
  int64_t blocks = (total + 7) / 8;
  const int64_t cap = static_cast<int64_t>(num_sms_of_current_device()) * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  LaunchScope scope(BWD ? HLM_KERNEL_QK_ROPE_BWD : HLM_KERNEL_QK_ROPE_FWD, s);
  qk_norm_rope_scalar_kernel<T, BWD><<<static_cast<int>(blocks), 256, 0, s>>>(
      static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(gq),
      static_cast<const T*>(gk), cosp, sinp, static_cast<T*>(q_out), static_cast<T*>(k_out), sh);
  return launch_status();
}

static int qk_common(bool bwd, const void* q, const void* k, const void* gq, const void* gk,
                     const void* cosp, const void* sinp, void* q_out, void* k_out, int64_t B,
                     int64_t T, int64_t Hq, int64_t Hk, int64_t D, int64_t rd,
                     const int64_t* q_strides, const int64_t* k_strides, int64_t cs_stride_t,
                     int cs_dtype, float eps, int dtype, void* stream) {
  if (B < 0 || T < 0 || Hq < 0 || Hk < 0 || D <= 0 || rd < 0 || rd > D || (rd & 1))
    return HLM_ERR_INVALID_ARG;
  if (q_strides == nullptr || k_strides == nullptr) return HLM_ERR_INVALID_ARG;
  if (cs_dtype != HLM_F32 && cs_dtype != HLM_BF16 && cs_dtype != HLM_F16)
    return HLM_ERR_UNSUPPORTED;
  if (B * T * (Hq + Hk) == 0) return HLM_OK;
  if (q == nullptr || k == nullptr || q_out == nullptr || k_out == nullptr)
    return HLM_ERR_INVALID_ARG;
  if (rd > 0 && (cosp == nullptr || sinp == nullptr)) return HLM_ERR_INVALID_ARG;
  if (bwd && (gq == nullptr || gk == nullptr)) return HLM_ERR_INVALID_ARG;
  QKShape sh;
  sh.B = B;
  sh.T = T;
  sh.Hq = Hq;
  sh.Hk = Hk;
  sh.D = D;
  sh.rd = rd;
  for (int i = 0; i < 4; ++i) {
    sh.qs[i] = q_strides[i];
    sh.ks[i] = k_strides[i];
  }
  sh.cs_stride = cs_stride_t;
  sh.cs_dtype = cs_dtype;
  sh.eps = eps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case HLM_F32:
      return bwd ? launch_qk_norm_rope<float, true>(q, k, gq, gk, cosp, sinp, q_out, k_out, sh, s)
                 : launch_qk_norm_rope<float, false>(q, k, gq, gk, cosp, sinp, q_out, k_out, sh, s);
    case HLM_BF16:
      return bwd ? launch_qk_norm_rope<__nv_bfloat16, true>(q, k, gq, gk, cosp, sinp, q_out,
                                                            k_out, sh, s)
                 : launch_qk_norm_rope<__nv_bfloat16, false>(q, k, gq, gk, cosp, sinp, q_out,
                                                             k_out, sh, s);
    case HLM_F16:
      return bwd ? launch_qk_norm_rope<__half, true>(q, k, gq, gk, cosp, sinp, q_out, k_out, sh, s)
                 : launch_qk_norm_rope<__half, false>(q, k, gq, gk, cosp, sinp, q_out, k_out, sh,
                                                      s);
    default:
      return HLM_ERR_UNSUPPORTED;
  }
}

}  // namespace hlm

extern "C" int hlm_qk_norm_rope_fwd(const void* q, const void* k, const void* cos, const void* sin,
                                    void* q_out, void* k_out, int64_t B, int64_t T, int64_t Hq,
                                    int64_t Hk, int64_t D, int64_t rotary_dim,
                                    const int64_t* q_strides, const int64_t* k_strides,
                                    int64_t cs_stride_t, int cs_dtype, float eps, int dtype,
                                    void* stream) {
  return hlm::qk_common(false, q, k, nullptr, nullptr, cos, sin, q_out, k_out, B, T, Hq, Hk, D,
                        rotary_dim, q_strides, k_strides, cs_stride_t, cs_dtype, eps, dtype,
                        stream);
}

extern "C" int hlm_qk_norm_rope_bwd(const void* q, const void* k, const void* grad_q,
                                    const void* grad_k, const void* cos, const void* sin,
                                    void* grad_q_in, void* grad_k_in, int64_t B, int64_t T,
                                    int64_t Hq, int64_t Hk, int64_t D, int64_t rotary_dim,
                                    const int64_t* q_strides, const int64_t* k_strides,
                                    int64_t cs_stride_t, int cs_dtype, float eps, int dtype,
                                    void* stream) {
  return hlm::qk_common(true, q, k, grad_q, grad_k, cos, sin, grad_q_in, grad_k_in, B, T, Hq, Hk,
                        D, rotary_dim, q_strides, k_strides, cs_stride_t, cs_dtype, eps, dtype,
                        stream);
}
