// QK-norm + partial rotate-half RoPE, forward and backward, on strided q/k
// views (the packed qkv GEMM output viewed as [B,T,H,D] with row stride
// (Hq+2Hk)*D).  Semantics follow kernels.py:446-503 (forward) and
// kernels.py:546-612 (backward):
//   forward : z = x*rsqrt(mean(x^2)+eps); rotate the first rotary_dim dims of
//             z with cos/sin[t, d mod half]; pass-through dims are z.
//   backward: g_n = inverse rotation of g; dx = inv*(g_n - z*mean(g_n*z)).
//
// Vector path: one head vector is spread over LPH lanes, each lane holding two
// 16-byte chunks chosen so that it owns whole rotation pairs (no partner
// loads); a warp walks the heads of one token at a time.  The sum of squares
// and the backward dot product are shuffle-xor reductions inside the LPH-lane
// group.
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

// A 16-byte chunk of T as float pairs (element 2j in .x, 2j+1 in .y), for the
// packed fp32x2 arithmetic of sm_100.
template <typename T>
struct Chunk {
  static constexpr int NP = 8 / sizeof(T);  // float pairs per chunk
  static HLM_DEVICE void unpack(const uint4& r, float2 (&f)[NP]) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
    if constexpr (std::is_same<T, float>::value) {
      f[0] = make_float2(__uint_as_float(w[0]), __uint_as_float(w[1]));
      f[1] = make_float2(__uint_as_float(w[2]), __uint_as_float(w[3]));
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        f[j] = make_float2(__uint_as_float(w[j] << 16), __uint_as_float(w[j] & 0xffff0000u));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) f[j] = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
    }
  }
  static HLM_DEVICE uint4 pack(const float2 (&f)[NP]) {
    uint32_t w[4];
    if constexpr (std::is_same<T, float>::value) {
      w[0] = __float_as_uint(f[0].x);
      w[1] = __float_as_uint(f[0].y);
      w[2] = __float_as_uint(f[1].x);
      w[3] = __float_as_uint(f[1].y);
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
      for (int j = 0; j < 4; ++j) w[j] = pack_bf16x2(f[j].x, f[j].y);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 h = __floats2half2_rn(f[j].x, f[j].y);
        w[j] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
};

HLM_DEVICE float rsqrt_ftz(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Token-major vector kernel.  A warp owns one token at a time and walks its
// H = Hq + Hk head vectors HPW = 32/LPH at a time, LPH = D / (2*CH) lanes per
// head vector, CH = 16/sizeof(T) elements per 16-byte chunk.  Every lane holds
// two chunks, laid out so that each lane owns whole rotation pairs:
//   rotated lane i < rd/(2*CH): dims [i*CH, +CH) and their partners [rd/2 + i*CH, +CH)
//   pass-through lane j:        dims [rd + j*CH, +CH) and [rd + (D-rd)/2 + j*CH, +CH)
// so the rotation needs no partner load and one branch-free formula serves
// every lane:
//   out0 = inv * (x0*c + s0*x1),  out1 = inv * (x1*c + s1*x0)
// with (c, s0, s1) = (cos, -sin, +sin) on rotated lanes and (1, 0, 0) on
// pass-through lanes (the inverse rotation of the backward flips the signs).
// Each load instruction of the warp covers whole 32-byte sectors.  The token's
// cos/sin slice and the (batch, position) index are computed once per token;
// U passes of loads are issued before any of them is used; the fp32 arithmetic
// runs on float pairs (fma.rn.f32x2 / mul.rn.f32x2, same rounding as scalar).
// Modes: kRopeFwd (x -> rotated norm), kRopeBwdX (x, g -> dx),
//        kRopeBwdY (saved output y, saved 1/rms, g -> dx; the normalised
//        vector z is the inverse rotation of y).
template <typename T, typename CS, int LPH, int MODE, int U>
HLM_DEVICE void qk_norm_rope_vec_body(const RopeArgs& a) {
  using C = Chunk<T>;
  constexpr int CH = 16 / sizeof(T);
  constexpr int NP = C::NP;
  constexpr int HPW = 32 / LPH;
  const int lane = threadIdx.x & 31;
  const int slot = lane / LPH, li = lane % LPH;
  const int H = a.Hq + a.Hk;
  const int Hq = a.Hq;
  const int D = a.D;
  const int half = a.rd >> 1;
  const int nrot = half / CH;
  const bool rot = li < nrot;
  const int off0 = rot ? li * CH : a.rd + (li - nrot) * CH;
  const int off1 = off0 + (rot ? half : (D - a.rd) >> 1);
  // sign of sin in the chunk-0 term: -1 forward, +1 for the inverse rotation
  const float sg = rot ? (MODE == kRopeFwd ? -1.0f : 1.0f) : 0.0f;
  const float crot = rot ? 1.0f : 0.0f;
  const float inv_d = 1.0f / static_cast<float>(D);
  const T* xq = static_cast<const T*>(a.xq);
  const T* xk = static_cast<const T*>(a.xk);
  const int passes = (H + HPW - 1) / HPW;
  const uint32_t nwarps = gridDim.x * (blockDim.x >> 5);
  uint32_t tok = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (tok >= a.tokens) return;
  // (batch, position) of the token, advanced by nwarps tokens per iteration
  uint32_t b = tok / a.T, t = tok - b * a.T;
  const uint32_t db = nwarps / a.T, dt = nwarps - db * a.T;
  for (; tok < a.tokens; tok += nwarps) {
    float2 c[NP], s0[NP], s1[NP];
    {
      float cf[CH], sf[CH];
      if (a.rd > 0) {
        const int64_t ci = static_cast<int64_t>(t) * a.cs_stride + (rot ? li * CH : 0);
        load_cs_vec<CS, CH>(static_cast<const CS*>(a.cosp) + ci, cf);
        load_cs_vec<CS, CH>(static_cast<const CS*>(a.sinp) + ci, sf);
      } else {
#pragma unroll
        for (int i = 0; i < CH; ++i) cf[i] = sf[i] = 0.0f;
      }
#pragma unroll
      for (int j = 0; j < NP; ++j) {
        c[j] = make_float2(fmaf(crot, cf[2 * j], 1.0f - crot), fmaf(crot, cf[2 * j + 1], 1.0f - crot));
        s0[j] = make_float2(sg * sf[2 * j], sg * sf[2 * j + 1]);
        s1[j] = make_float2(-s0[j].x, -s0[j].y);
      }
    }
    const T* qrow = xq + b * a.qs0 + t * a.qs1;
    const T* krow = xk + b * a.ks0 + t * a.ks1;
    const int64_t qo = static_cast<int64_t>(tok) * Hq * D;  // outputs / grads: contiguous
    const int64_t ko = static_cast<int64_t>(tok) * a.Hk * D;
    for (int p0 = 0; p0 < passes; p0 += U) {
      uint4 r0[U], r1[U], gr0[U], gr1[U];
      float rs[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int h = (p0 + u) * HPW + slot;
        const int hc = h < H ? h : 0;
        const bool is_q = hc < Hq;
        const int hh = is_q ? hc : hc - Hq;
        const T* row = is_q ? qrow + hh * a.qs2 : krow + hh * a.ks2;
        r0[u] = ld_global_nc_v4(row + off0);
        r1[u] = ld_global_nc_v4(row + off1);
        if constexpr (MODE != kRopeFwd) {
          const T* grow = static_cast<const T*>(is_q ? a.gq : a.gk) + (is_q ? qo : ko) +
                          static_cast<int64_t>(hh) * D;
          gr0[u] = ld_global_nc_v4(grow + off0);
          gr1[u] = ld_global_nc_v4(grow + off1);
        }
        if constexpr (MODE == kRopeBwdY) rs[u] = a.rstd[static_cast<int64_t>(tok) * H + hc];
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int h = (p0 + u) * HPW + slot;
        float2 x0[NP], x1[NP], o0[NP], o1[NP];
        C::unpack(r0[u], x0);
        C::unpack(r1[u], x1);
        if constexpr (MODE == kRopeFwd) {
          float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < NP; ++j) acc = __ffma2_rn(x0[j], x0[j], acc);
#pragma unroll
          for (int j = 0; j < NP; ++j) acc = __ffma2_rn(x1[j], x1[j], acc);
          const float ss = group_sum<LPH>(acc.x + acc.y);
          const float inv = rsqrt_ftz(fmaf(ss, inv_d, a.eps));
          const float2 inv2 = make_float2(inv, inv);
#pragma unroll
          for (int j = 0; j < NP; ++j) {
            o0[j] = __fmul2_rn(inv2, __ffma2_rn(s0[j], x1[j], __fmul2_rn(x0[j], c[j])));
            o1[j] = __fmul2_rn(inv2, __ffma2_rn(s1[j], x0[j], __fmul2_rn(x1[j], c[j])));
          }
        } else {
          float2 g0[NP], g1[NP], z0[NP], z1[NP];
          C::unpack(gr0[u], g0);
          C::unpack(gr1[u], g1);
          float inv;
          if constexpr (MODE == kRopeBwdX) {
            float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int j = 0; j < NP; ++j) acc = __ffma2_rn(x0[j], x0[j], acc);
#pragma unroll
            for (int j = 0; j < NP; ++j) acc = __ffma2_rn(x1[j], x1[j], acc);
            const float ss = group_sum<LPH>(acc.x + acc.y);
            inv = rsqrt_ftz(fmaf(ss, inv_d, a.eps));
            const float2 inv2 = make_float2(inv, inv);
#pragma unroll
            for (int j = 0; j < NP; ++j) {
              z0[j] = __fmul2_rn(x0[j], inv2);
              z1[j] = __fmul2_rn(x1[j], inv2);
            }
          } else {
            inv = rs[u];
            // inverse rotation of the saved output y gives the normalised vector
#pragma unroll
            for (int j = 0; j < NP; ++j) {
              z0[j] = __ffma2_rn(s0[j], x1[j], __fmul2_rn(x0[j], c[j]));
              z1[j] = __ffma2_rn(s1[j], x0[j], __fmul2_rn(x1[j], c[j]));
            }
          }
          // inverse rotation of the output gradient (into g0 / g1), then mean(g_n * z)
          float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < NP; ++j) {
            const float2 n0 = __ffma2_rn(s0[j], g1[j], __fmul2_rn(g0[j], c[j]));
            const float2 n1 = __ffma2_rn(s1[j], g0[j], __fmul2_rn(g1[j], c[j]));
            g0[j] = n0;
            g1[j] = n1;
            acc = __ffma2_rn(n0, z0[j], acc);
            acc = __ffma2_rn(n1, z1[j], acc);
          }
          const float ndot = -group_sum<LPH>(acc.x + acc.y) * inv_d;
          const float2 nd2 = make_float2(ndot, ndot), inv2 = make_float2(inv, inv);
#pragma unroll
          for (int j = 0; j < NP; ++j) {
            o0[j] = __fmul2_rn(inv2, __ffma2_rn(z0[j], nd2, g0[j]));
            o1[j] = __fmul2_rn(inv2, __ffma2_rn(z1[j], nd2, g1[j]));
          }
        }
        if (h < H) {
          const bool is_q = h < Hq;
          const int hh = is_q ? h : h - Hq;
          T* orow = static_cast<T*>(is_q ? a.oq : a.ok) + (is_q ? qo : ko) +
                    static_cast<int64_t>(hh) * D;
          st_global_v4(orow + off0, C::pack(o0));
          st_global_v4(orow + off1, C::pack(o1));
        }
      }
    }
    t += dt;
    b += db;
    if (t >= a.T) {
      t -= a.T;
      ++b;
    }
  }
}

// The forward is held to 85 registers (three 256-thread blocks per SM: more
// loads in flight, measured 10% faster); the backward keeps its registers.
template <typename T, typename CS, int LPH, int U>
__global__ void __launch_bounds__(256, 3) qk_norm_rope_fwd_vec_kernel(const RopeArgs a) {
  qk_norm_rope_vec_body<T, CS, LPH, kRopeFwd, U>(a);
}
template <typename T, typename CS, int LPH, int MODE, int U>
__global__ void __launch_bounds__(256) qk_norm_rope_bwd_vec_kernel(const RopeArgs a) {
  qk_norm_rope_vec_body<T, CS, LPH, MODE, U>(a);
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
  void (*kern)(const RopeArgs);
  if constexpr (MODE == kRopeFwd)
    kern = qk_norm_rope_fwd_vec_kernel<T, CS, LPH, U>;
  else
    kern = qk_norm_rope_bwd_vec_kernel<T, CS, LPH, MODE, U>;
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
    case 4:
      launch_rope_vec_lph<T, CS, 4, MODE>(a, warps_needed, s);
      break;
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
  constexpr int CH = 16 / sizeof(T);  // elements per 16-byte chunk, two chunks per lane
  const int lph = a.D / (2 * CH);
  bool vec = a.D % (2 * CH) == 0 && (lph == 4 || lph == 8 || lph == 16 || lph == 32);
  vec = vec && (a.rd / 2) % CH == 0 && a.rd <= a.D;
  const int64_t strides[] = {a.qs0, a.qs1, a.qs2, a.ks0, a.ks1, a.ks2};
  for (int64_t st : strides) vec = vec && st % CH == 0;
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
