// QK-norm + partial rotate-half RoPE, forward and backward, on strided q/k
// views (the packed qkv GEMM output viewed as [B,T,H,D] with row stride
// (Hq+2Hk)*D).  Semantics follow kernels.py:446-503 (forward) and
// kernels.py:546-612 (backward):
//   forward : z = x*rsqrt(mean(x^2)+eps); rotate the first rotary_dim dims of
//             z with cos/sin[t, d mod half]; pass-through dims are z.
//   backward: g_n = inverse rotation of g; dx = inv*(g_n - z*mean(g_n*z)).
//
// Vector path: one head vector is spread over LPH = D/VEC lanes, each lane
// holding one 16-byte vector.  The rotation partner of a lane's vector sits
// `half/VEC` lanes away and is fetched with a shuffle instead of being
// re-read from memory; the sum of squares and the backward dot product are
// shuffle-xor reductions inside the LPH-lane group.
#include <type_traits>

#include "hlm_common.cuh"

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

// One warp per token: the warp's LPH-lane groups take head vectors
// h = j*HPW + group for j < J, covering all Hq+Hk heads of q then k.  A lane
// keeps the same dims d0..d0+VEC-1 for every head, so its cos/sin values are
// loaded once per token, and all J head loads (2J in the backward) are issued
// before any math so each lane has J independent 16-byte loads in flight.
template <typename T, typename CS, int LPH, bool BWD, int J>
__global__ void __launch_bounds__(256) qk_norm_rope_vec_kernel(
    const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ gq,
    const T* __restrict__ gk, const CS* __restrict__ cosp, const CS* __restrict__ sinp,
    T* __restrict__ q_out, T* __restrict__ k_out, QKShape sh) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int HPW = 32 / LPH;  // head vectors per warp per j
  const int lane = threadIdx.x & 31;
  const int slot = lane / LPH;
  const int li = lane % LPH;
  const int H = static_cast<int>(sh.Hq + sh.Hk);
  const int Hq = static_cast<int>(sh.Hq);
  const uint32_t T_ = static_cast<uint32_t>(sh.T);
  const uint32_t tokens = static_cast<uint32_t>(sh.B * sh.T);
  const int half = static_cast<int>(sh.rd / 2);
  const int d0 = li * VEC;
  const int pdelta = half / VEC;  // lane distance of the rotation partner
  const int role = d0 < half ? 0 : (d0 < sh.rd ? 1 : 2);
  const int src_lane = role == 0 ? lane + pdelta : (role == 1 ? lane - pdelta : lane);
  const int cbase = role == 0 ? d0 : d0 - half;
  const float inv_d = 1.0f / static_cast<float>(sh.D);
  const uint32_t warps_total = gridDim.x * (blockDim.x >> 5);

  for (uint32_t tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); tok < tokens;
       tok += warps_total) {
    const uint32_t b = tok / T_;
    const uint32_t t = tok - b * T_;
    const int64_t qbase = b * sh.qs[0] + t * sh.qs[1] + d0;
    const int64_t kbase = b * sh.ks[0] + t * sh.ks[1] + d0;
    uint4 xraw[J], graw[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int h = j * HPW + slot;
      xraw[j] = make_uint4(0, 0, 0, 0);
      graw[j] = make_uint4(0, 0, 0, 0);
      if (h < H) {
        const bool is_q = h < Hq;
        const int hh = is_q ? h : h - Hq;
        xraw[j] = ld_global_nc_v4(is_q ? q + qbase + hh * sh.qs[2] : k + kbase + hh * sh.ks[2]);
        if constexpr (BWD) {
          const int64_t off = (static_cast<int64_t>(tok) * (is_q ? sh.Hq : sh.Hk) + hh) * sh.D + d0;
          graw[j] = ld_global_nc_v4((is_q ? gq : gk) + off);
        }
      }
    }
    float c[VEC], s[VEC];
    if (role != 2) {
      load_cs_vec<CS, VEC>(cosp + t * sh.cs_stride + cbase, c);
      load_cs_vec<CS, VEC>(sinp + t * sh.cs_stride + cbase, s);
    } else {
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        c[i] = 1.0f;
        s[i] = 0.0f;
      }
    }
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int h = j * HPW + slot;
      float x[VEC];
      Vec16<T> xv;
      xv.raw = xraw[j];
      xv.to_float(x);
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) ss += x[i] * x[i];
      ss = group_sum<LPH>(ss);
      const float inv = rsqrtf(ss * inv_d + sh.eps);
      float res[VEC];
      if constexpr (!BWD) {
        float z[VEC], pz[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) z[i] = x[i] * inv;
#pragma unroll
        for (int i = 0; i < VEC; ++i) pz[i] = __shfl_sync(0xffffffffu, z[i], src_lane);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          res[i] = role == 0 ? z[i] * c[i] - pz[i] * s[i]
                             : (role == 1 ? z[i] * c[i] + pz[i] * s[i] : z[i]);
        }
      } else {
        float g[VEC], pg[VEC], gn[VEC];
        Vec16<T> gv;
        gv.raw = graw[j];
        gv.to_float(g);
#pragma unroll
        for (int i = 0; i < VEC; ++i) pg[i] = __shfl_sync(0xffffffffu, g[i], src_lane);
        float dot = 0.0f;
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          gn[i] = role == 0 ? g[i] * c[i] + pg[i] * s[i]
                            : (role == 1 ? g[i] * c[i] - pg[i] * s[i] : g[i]);
          dot += gn[i] * x[i] * inv;
        }
        dot = group_sum<LPH>(dot) * inv_d;
#pragma unroll
        for (int i = 0; i < VEC; ++i) res[i] = inv * (gn[i] - x[i] * inv * dot);
      }
      if (h < H) {
        const bool is_q = h < Hq;
        const int hh = is_q ? h : h - Hq;
        const int64_t off = (static_cast<int64_t>(tok) * (is_q ? sh.Hq : sh.Hk) + hh) * sh.D + d0;
        Vec16<T> ov;
        ov.from_float(res);
        st_global_v4((is_q ? q_out : k_out) + off, ov.raw);
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

template <typename T, typename CS, int LPH, bool BWD, int J>
static void launch_qk_vec(const void* q, const void* k, const void* gq, const void* gk,
                          const void* cosp, const void* sinp, void* q_out, void* k_out,
                          const QKShape& sh, int blocks, cudaStream_t s) {
  qk_norm_rope_vec_kernel<T, CS, LPH, BWD, J><<<blocks, 256, 0, s>>>(
      static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(gq),
      static_cast<const T*>(gk), static_cast<const CS*>(cosp), static_cast<const CS*>(sinp),
      static_cast<T*>(q_out), static_cast<T*>(k_out), sh);
}

template <typename T, typename CS, int LPH, bool BWD>
static void launch_qk_vec_j(int j, const void* q, const void* k, const void* gq, const void* gk,
                            const void* cosp, const void* sinp, void* q_out, void* k_out,
                            const QKShape& sh, int blocks, cudaStream_t s) {
  if (j <= 2)
    launch_qk_vec<T, CS, LPH, BWD, 2>(q, k, gq, gk, cosp, sinp, q_out, k_out, sh, blocks, s);
  else if (j <= 4)
    launch_qk_vec<T, CS, LPH, BWD, 4>(q, k, gq, gk, cosp, sinp, q_out, k_out, sh, blocks, s);
  else if (j <= 6)
    launch_qk_vec<T, CS, LPH, BWD, 6>(q, k, gq, gk, cosp, sinp, q_out, k_out, sh, blocks, s);
  else
    launch_qk_vec<T, CS, LPH, BWD, 8>(q, k, gq, gk, cosp, sinp, q_out, k_out, sh, blocks, s);
}

template <typename T, bool BWD>
static int launch_qk_norm_rope(const void* q, const void* k, const void* gq, const void* gk,
                               const void* cosp, const void* sinp, void* q_out, void* k_out,
                               const QKShape& sh, cudaStream_t s) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t tokens = sh.B * sh.T;
  const int64_t total = tokens * (sh.Hq + sh.Hk);
  const int64_t lph = sh.D / VEC;
  const bool cs_same = (sh.cs_dtype == HLM_F32 && sizeof(T) == 4) ||
                       (sh.cs_dtype == HLM_BF16 && std::is_same<T, __nv_bfloat16>::value) ||
                       (sh.cs_dtype == HLM_F16 && std::is_same<T, __half>::value);
  const bool cs_f32 = sh.cs_dtype == HLM_F32;
  const int cs_size = cs_f32 ? 4 : 2;
  bool vec = sh.D % VEC == 0 && (lph == 8 || lph == 16 || lph == 32);
  const int64_t hpw = lph > 0 ? 32 / lph : 0;
  const int64_t jneed = hpw > 0 ? (sh.Hq + sh.Hk + hpw - 1) / hpw : 0;
  vec = vec && jneed <= 8;
  vec = vec && (sh.rd / 2) % VEC == 0 && sh.qs[3] == 1 && sh.ks[3] == 1;
  for (int i = 0; i < 3; ++i) vec = vec && sh.qs[i] % VEC == 0 && sh.ks[i] % VEC == 0;
  vec = vec && host_aligned16(q) && host_aligned16(k) && host_aligned16(q_out) &&
        host_aligned16(k_out);
  if (BWD) vec = vec && host_aligned16(gq) && host_aligned16(gk);
  vec = vec && (cs_same || cs_f32) && tokens < (1ll << 31);
  if (sh.rd > 0)
    vec = vec && host_aligned16(cosp) && host_aligned16(sinp) && (sh.cs_stride * cs_size) % 16 == 0;
  const int threads = 256;
  LaunchScope scope(BWD ? HLM_KERNEL_QK_ROPE_BWD : HLM_KERNEL_QK_ROPE_FWD, s);
  if (vec) {
    int64_t blocks = (tokens + 7) / 8;  // one warp per token
    const int64_t cap = static_cast<int64_t>(num_sms_of_current_device()) * 64;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    const int nb = static_cast<int>(blocks);
    const int j = static_cast<int>(jneed);
#define HLM_QK_CS(CS)                                                                          \
  switch (lph) {                                                                               \
    case 8: launch_qk_vec_j<T, CS, 8, BWD>(j, q, k, gq, gk, cosp, sinp, q_out, k_out, sh, nb, s); break; \
    case 16: launch_qk_vec_j<T, CS, 16, BWD>(j, q, k, gq, gk, cosp, sinp, q_out, k_out, sh, nb, s); break; \
    default: launch_qk_vec_j<T, CS, 32, BWD>(j, q, k, gq, gk, cosp, sinp, q_out, k_out, sh, nb, s); break; \
  }
    if (cs_f32) {
      HLM_QK_CS(float)
    } else {
      HLM_QK_CS(T)
    }
#undef HLM_QK_CS
  } else {
    int64_t blocks = (total + 7) / 8;
    const int64_t cap = static_cast<int64_t>(num_sms_of_current_device()) * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    qk_norm_rope_scalar_kernel<T, BWD><<<static_cast<int>(blocks), threads, 0, s>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(gq),
        static_cast<const T*>(gk), cosp, sinp, static_cast<T*>(q_out), static_cast<T*>(k_out),
        sh);
  }
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
