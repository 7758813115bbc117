// Memory-bound operators of the hackable-lm hot path: SwiGLU forward/backward,
// residual-add + RMSNorm forward/backward (optional weight), and the scalar
// rescale used by the fused LM-head backward.
//
// Design: 128-bit vectorised coalesced loads (ld.global.nc for streamed
// inputs), fp32 math in registers, one warp per row for the row reductions
// (shuffle-xor trees, no shared memory), grids sized to the SM count.  A
// scalar path covers shapes whose rows are not 16-byte multiples (the
// reference accepts any even width, e.g. the [17,130] fp32 GPU test).
#include <mutex>

#include "hlm_common.cuh"

namespace hlm {

template <typename T>
struct DTypeOf;
template <>
struct DTypeOf<float> {
  static constexpr int value = HLM_F32;
};
template <>
struct DTypeOf<__nv_bfloat16> {
  static constexpr int value = HLM_BF16;
};
template <>
struct DTypeOf<__half> {
  static constexpr int value = HLM_F16;
};

#define HLM_DISPATCH_DTYPE(dtype, T, ...)          \
  switch (dtype) {                                 \
    case HLM_F32: {                                \
      using T = float;                             \
      __VA_ARGS__;                                 \
      break;                                       \
    }                                              \
    case HLM_BF16: {                               \
      using T = __nv_bfloat16;                     \
      __VA_ARGS__;                                 \
      break;                                       \
    }                                              \
    case HLM_F16: {                                \
      using T = __half;                            \
      __VA_ARGS__;                                 \
      break;                                       \
    }                                              \
    default:                                       \
      return HLM_ERR_UNSUPPORTED;                  \
  }

static inline int elementwise_grid(int64_t work_items, int threads) {
  const int64_t max_blocks = static_cast<int64_t>(num_sms_of_current_device()) * (2048 / threads);
  int64_t blocks = (work_items + threads - 1) / threads;
  if (blocks > max_blocks) blocks = max_blocks;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

// Grid for row-oriented kernels: enough blocks to cover every row group once,
// capped at a multiple of the SM count for very tall inputs.
static inline int rows_grid(int64_t rows, int rows_per_block) {
  const int64_t cap = static_cast<int64_t>(num_sms_of_current_device()) * 64;
  int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

// ---------------------------------------------------------------------------
// SwiGLU (kernels.py:343-386)
// ---------------------------------------------------------------------------
// Row-oriented: a block owns R consecutive rows per iteration and its threads
// stride over the 16-byte vectors of each half-row, so every thread keeps 2*R
// independent 16-byte loads in flight and no index division is needed.
template <typename T, int R>
__global__ void __launch_bounds__(256) swiglu_fwd_vec_kernel(const T* __restrict__ gate_up,
                                                            T* __restrict__ out, int64_t rows,
                                                            int hv) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t hidden = static_cast<int64_t>(hv) * VEC;
  for (int64_t r0 = static_cast<int64_t>(blockIdx.x) * R; r0 < rows;
       r0 += static_cast<int64_t>(gridDim.x) * R) {
    for (int cv = threadIdx.x; cv < hv; cv += blockDim.x) {
      uint4 g_raw[R], u_raw[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r0 + r < rows) {
          const T* src = gate_up + (r0 + r) * 2 * hidden + static_cast<int64_t>(cv) * VEC;
          g_raw[r] = ld_global_nc_v4(src);
          u_raw[r] = ld_global_nc_v4(src + hidden);
        }
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r0 + r >= rows) continue;
        Vec16<T> gv, uv, ov;
        gv.raw = g_raw[r];
        uv.raw = u_raw[r];
        float g[VEC], up[VEC], o[VEC];
        gv.to_float(g);
        uv.to_float(up);
#pragma unroll
        for (int i = 0; i < VEC; ++i) o[i] = g[i] * sigmoid_fast(g[i]) * up[i];
        ov.from_float(o);
        st_global_v4(out + (r0 + r) * hidden + static_cast<int64_t>(cv) * VEC, ov.raw);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_fwd_scalar_kernel(const T* __restrict__ gate_up,
                                                               T* __restrict__ out, int64_t rows,
                                                               int64_t hidden) {
  const int64_t total = rows * hidden;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / hidden, col = i - row * hidden;
    const float g = to_f32(gate_up[row * 2 * hidden + col]);
    const float u = to_f32(gate_up[row * 2 * hidden + hidden + col]);
    out[i] = from_f32<T>(g * sigmoidf_(g) * u);
  }
}

template <typename T, int R>
__global__ void __launch_bounds__(256) swiglu_bwd_vec_kernel(const T* __restrict__ gate_up,
                                                            const T* __restrict__ grad_out,
                                                            T* __restrict__ grad_gate_up,
                                                            int64_t rows, int hv) {
  constexpr int VEC = 16 / sizeof(T);
  const int64_t hidden = static_cast<int64_t>(hv) * VEC;
  for (int64_t r0 = static_cast<int64_t>(blockIdx.x) * R; r0 < rows;
       r0 += static_cast<int64_t>(gridDim.x) * R) {
    for (int cv = threadIdx.x; cv < hv; cv += blockDim.x) {
      uint4 g_raw[R], u_raw[R], d_raw[R];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r0 + r < rows) {
          const int64_t off_in = (r0 + r) * 2 * hidden + static_cast<int64_t>(cv) * VEC;
          g_raw[r] = ld_global_nc_v4(gate_up + off_in);
          u_raw[r] = ld_global_nc_v4(gate_up + off_in + hidden);
          d_raw[r] = ld_global_nc_v4(grad_out + (r0 + r) * hidden + static_cast<int64_t>(cv) * VEC);
        }
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r0 + r >= rows) continue;
        Vec16<T> gv, uv, dv, og, ou;
        gv.raw = g_raw[r];
        uv.raw = u_raw[r];
        dv.raw = d_raw[r];
        float g[VEC], up[VEC], d[VEC], rg[VEC], ru[VEC];
        gv.to_float(g);
        uv.to_float(up);
        dv.to_float(d);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const float sg = sigmoid_fast(g[i]);
          const float silu = g[i] * sg;
          const float dsilu = sg * (1.0f + g[i] * (1.0f - sg));
          rg[i] = d[i] * up[i] * dsilu;
          ru[i] = d[i] * silu;
        }
        og.from_float(rg);
        ou.from_float(ru);
        const int64_t off_in = (r0 + r) * 2 * hidden + static_cast<int64_t>(cv) * VEC;
        st_global_v4(grad_gate_up + off_in, og.raw);
        st_global_v4(grad_gate_up + off_in + hidden, ou.raw);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_bwd_scalar_kernel(const T* __restrict__ gate_up,
                                                               const T* __restrict__ grad_out,
                                                               T* __restrict__ grad_gate_up,
                                                               int64_t rows, int64_t hidden) {
  const int64_t total = rows * hidden;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / hidden, col = i - row * hidden;
    const int64_t gi = row * 2 * hidden + col;
    const float g = to_f32(gate_up[gi]);
    const float u = to_f32(gate_up[gi + hidden]);
    const float d = to_f32(grad_out[i]);
    const float s = sigmoidf_(g);
    grad_gate_up[gi] = from_f32<T>(d * u * s * (1.0f + g * (1.0f - s)));
    grad_gate_up[gi + hidden] = from_f32<T>(d * g * s);
  }
}

// ---------------------------------------------------------------------------
// Residual add + RMSNorm (model.py:14-16, 73-75)
// One warp per row; lane l owns 16-byte vectors l, l+32, ... of the row.
// ---------------------------------------------------------------------------
template <typename T, int NV>
__global__ void __launch_bounds__(256) rmsnorm_fwd_vec_kernel(
    const T* __restrict__ residual, const T* __restrict__ branch, const T* __restrict__ weight,
    T* __restrict__ out, T* __restrict__ norm, int64_t rows, int cols, float eps) {
  constexpr int VEC = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const float inv_cols = 1.0f / static_cast<float>(cols);
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); row < rows;
       row += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t base = row * cols;
    uint4 braw[NV], rraw[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * VEC;
      if (c < cols) {
        braw[j] = ld_global_nc_v4(branch + base + c);
        if (residual != nullptr) rraw[j] = ld_global_nc_v4(residual + base + c);
      }
    }
    float x[NV][VEC];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * VEC;
      if (c < cols) {
        Vec16<T> bv;
        bv.raw = braw[j];
        bv.to_float(x[j]);
        if (residual != nullptr) {
          Vec16<T> rv, ov;
          rv.raw = rraw[j];
          float r[VEC];
          rv.to_float(r);
#pragma unroll
          for (int i = 0; i < VEC; ++i) x[j][i] += r[i];
          ov.from_float(x[j]);
          st_global_v4(out + base + c, ov.raw);
          ov.to_float(x[j]);  // the norm sees the value stored in `out` (dtype-rounded)
        }
#pragma unroll
        for (int i = 0; i < VEC; ++i) ss += x[j][i] * x[j][i];
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss * inv_cols + eps);
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * VEC;
      if (c < cols) {
        float y[VEC];
        if (weight != nullptr) {
          Vec16<T> wv;
          wv.raw = ld_global_v4(weight + c);
          float w[VEC];
          wv.to_float(w);
#pragma unroll
          for (int i = 0; i < VEC; ++i) y[i] = x[j][i] * r * w[i];
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) y[i] = x[j][i] * r;
        }
        Vec16<T> yv;
        yv.from_float(y);
        st_global_v4(norm + base + c, yv.raw);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_fwd_scalar_kernel(
    const T* __restrict__ residual, const T* __restrict__ branch, const T* __restrict__ weight,
    T* __restrict__ out, T* __restrict__ norm, int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); row < rows;
       row += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t base = row * cols;
    float ss = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      float x = to_f32(branch[base + c]);
      if (residual != nullptr) {
        const T o = from_f32<T>(x + to_f32(residual[base + c]));
        out[base + c] = o;
        x = to_f32(o);
      }
      ss += x * x;
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(cols) + eps);
    __syncwarp();
    for (int c = lane; c < cols; c += 32) {
      const float x = residual != nullptr ? to_f32(out[base + c]) : to_f32(branch[base + c]);
      float y = x * r;
      if (weight != nullptr) y *= to_f32(weight[c]);
      norm[base + c] = from_f32<T>(y);
    }
  }
}

// Backward.  With HAS_W, partial receives per-warp sums of g*x*r for dweight:
// partial[(blockIdx.x * wpb + warp) * cols + c].  Without a weight the
// kernel keeps no weight or dweight registers (the model's norms are
// weightless), which keeps occupancy high.
template <typename T, int NV, bool HAS_W>
__global__ void __launch_bounds__(256) rmsnorm_bwd_vec_kernel(
    const T* __restrict__ xin, const T* __restrict__ weight, const T* __restrict__ grad_out,
    const T* __restrict__ grad_norm, T* __restrict__ grad_in, float* __restrict__ partial,
    int64_t rows, int cols, float eps) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int NW = HAS_W ? NV : 1;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const float inv_cols = 1.0f / static_cast<float>(cols);
  float wacc[NW][VEC];
  float w[NW][VEC];
  if constexpr (HAS_W) {
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * VEC;
#pragma unroll
      for (int i = 0; i < VEC; ++i) {
        wacc[j][i] = 0.0f;
        w[j][i] = 1.0f;
      }
      if (c < cols) {
        Vec16<T> wv;
        wv.raw = ld_global_v4(weight + c);
        wv.to_float(w[j]);
      }
    }
  }
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); row < rows;
       row += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t base = row * cols;
    uint4 xraw[NV], graw[NV], oraw[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * VEC;
      if (c < cols) {
        xraw[j] = ld_global_nc_v4(xin + base + c);
        graw[j] = ld_global_nc_v4(grad_norm + base + c);
        if (grad_out != nullptr) oraw[j] = ld_global_nc_v4(grad_out + base + c);
      }
    }
    float ss = 0.0f, dot = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * VEC;
      if (c < cols) {
        Vec16<T> xv, gv;
        xv.raw = xraw[j];
        gv.raw = graw[j];
        float x[VEC], g[VEC];
        xv.to_float(x);
        gv.to_float(g);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          ss += x[i] * x[i];
          const float gw = HAS_W ? g[i] * w[HAS_W ? j : 0][i] : g[i];
          dot += gw * x[i];
        }
      }
    }
    ss = warp_sum(ss);
    dot = warp_sum(dot);
    const float r = rsqrtf(ss * inv_cols + eps);
    const float k3 = r * r * r * dot * inv_cols;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * VEC;
      if (c < cols) {
        Vec16<T> xv, gv;
        xv.raw = xraw[j];
        gv.raw = graw[j];
        float x[VEC], g[VEC], go[VEC];
        xv.to_float(x);
        gv.to_float(g);
        if (grad_out != nullptr) {
          Vec16<T> ov;
          ov.raw = oraw[j];
          ov.to_float(go);
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) go[i] = 0.0f;
        }
        float d[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const float gw = HAS_W ? g[i] * w[HAS_W ? j : 0][i] : g[i];
          d[i] = go[i] + r * gw - x[i] * k3;
          if constexpr (HAS_W) wacc[j][i] += g[i] * x[i] * r;
        }
        Vec16<T> dv;
        dv.from_float(d);
        st_global_v4(grad_in + base + c, dv.raw);
      }
    }
  }
  if constexpr (HAS_W) {
    float* dst = partial + (static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5)) * cols;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int c = (lane + 32 * j) * VEC;
      if (c < cols) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) dst[c + i] = wacc[j][i];
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_bwd_scalar_kernel(
    const T* __restrict__ xin, const T* __restrict__ weight, const T* __restrict__ grad_out,
    const T* __restrict__ grad_norm, T* __restrict__ grad_in, float* __restrict__ partial,
    int64_t rows, int cols, float eps) {
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  float* dst = partial != nullptr
                   ? partial + (static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5)) * cols
                   : nullptr;
  if (dst != nullptr)
    for (int c = lane; c < cols; c += 32) dst[c] = 0.0f;
  for (int64_t row = static_cast<int64_t>(blockIdx.x) * wpb + (threadIdx.x >> 5); row < rows;
       row += static_cast<int64_t>(gridDim.x) * wpb) {
    const int64_t base = row * cols;
    float ss = 0.0f, dot = 0.0f;
    for (int c = lane; c < cols; c += 32) {
      const float x = to_f32(xin[base + c]);
      const float w = weight != nullptr ? to_f32(weight[c]) : 1.0f;
      ss += x * x;
      dot += to_f32(grad_norm[base + c]) * w * x;
    }
    ss = warp_sum(ss);
    dot = warp_sum(dot);
    const float r = rsqrtf(ss / static_cast<float>(cols) + eps);
    const float k3 = r * r * r * dot / static_cast<float>(cols);
    for (int c = lane; c < cols; c += 32) {
      const float x = to_f32(xin[base + c]);
      const float g = to_f32(grad_norm[base + c]);
      const float w = weight != nullptr ? to_f32(weight[c]) : 1.0f;
      const float go = grad_out != nullptr ? to_f32(grad_out[base + c]) : 0.0f;
      grad_in[base + c] = from_f32<T>(go + r * g * w - x * k3);
      if (dst != nullptr) dst[c] += g * x * r;
    }
  }
}

// grad_weight[c] = sum_p partial[p][c]  (fixed summation order: deterministic)
template <typename T>
__global__ void __launch_bounds__(256) reduce_partials_kernel(const float* __restrict__ partial,
                                                             T* __restrict__ grad_weight,
                                                             int num_partials, int cols) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float acc = 0.0f;
  for (int p = 0; p < num_partials; ++p) acc += partial[static_cast<int64_t>(p) * cols + c];
  grad_weight[c] = from_f32<T>(acc);
}

// data *= *scale
template <typename T>
__global__ void __launch_bounds__(256) scale_kernel(T* __restrict__ data,
                                                   const float* __restrict__ scale, int64_t n) {
  constexpr int VEC = 16 / sizeof(T);
  const float s = *scale;
  const int64_t nv = n / VEC;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int64_t v = tid; v < nv; v += stride) {
    Vec16<T> x;
    x.raw = ld_global_v4(data + v * VEC);
    float f[VEC];
    x.to_float(f);
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] *= s;
    x.from_float(f);
    st_global_v4(data + v * VEC, x.raw);
  }
  for (int64_t i = nv * VEC + tid; i < n; i += stride) data[i] = from_f32<T>(to_f32(data[i]) * s);
}

// Number of per-warp dweight partials used by the RMSNorm backward.
static constexpr int kRmsBwdThreads = 256;
static constexpr int kRmsBwdWarps = kRmsBwdThreads / 32;
static constexpr int kRmsBwdMaxBlocks = 128;

static inline int rms_bwd_weight_blocks(int64_t rows) {
  int64_t b = (rows + kRmsBwdWarps - 1) / kRmsBwdWarps;
  if (b > kRmsBwdMaxBlocks) b = kRmsBwdMaxBlocks;
  if (b < 1) b = 1;
  return static_cast<int>(b);
}

template <typename T>
static int pick_nv(int cols) {
  constexpr int VEC = 16 / sizeof(T);
  const int nv = (cols + 32 * VEC - 1) / (32 * VEC);
  if (nv <= 1) return 1;
  if (nv <= 2) return 2;
  if (nv <= 3) return 3;
  if (nv <= 4) return 4;
  if (nv <= 6) return 6;
  if (nv <= 8) return 8;
  return 0;  // too wide for the register-resident path
}

#define HLM_DISPATCH_NV(nv, NVC, ...) \
  switch (nv) {                       \
    case 1: {                         \
      constexpr int NVC = 1;          \
      __VA_ARGS__;                    \
      break;                          \
    }                                 \
    case 2: {                         \
      constexpr int NVC = 2;          \
      __VA_ARGS__;                    \
      break;                          \
    }                                 \
    case 3: {                         \
      constexpr int NVC = 3;          \
      __VA_ARGS__;                    \
      break;                          \
    }                                 \
    case 4: {                         \
      constexpr int NVC = 4;          \
      __VA_ARGS__;                    \
      break;                          \
    }                                 \
    case 6: {                         \
      constexpr int NVC = 6;          \
      __VA_ARGS__;                    \
      break;                          \
    }                                 \
    default: {                        \
      constexpr int NVC = 8;          \
      __VA_ARGS__;                    \
      break;                          \
    }                                 \
  }

}  // namespace hlm

using namespace hlm;

extern "C" int hlm_swiglu_fwd(const void* gate_up, void* out, int64_t rows, int64_t hidden,
                              int dtype, void* stream) {
  if (rows < 0 || hidden < 0) return HLM_ERR_INVALID_ARG;
  if (rows == 0 || hidden == 0) return HLM_OK;
  if (gate_up == nullptr || out == nullptr) return HLM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LaunchScope scope(HLM_KERNEL_SWIGLU_FWD, s);
  HLM_DISPATCH_DTYPE(dtype, T, {
    constexpr int VEC = 16 / sizeof(T);
    const bool vec = (hidden % VEC == 0) && host_aligned16(gate_up) && host_aligned16(out);
    if (vec && hidden / VEC <= (1ll << 30)) {
      constexpr int R = 4;
      const int grid = rows_grid(rows, R);
      swiglu_fwd_vec_kernel<T, R><<<grid, 256, 0, s>>>(static_cast<const T*>(gate_up),
                                                       static_cast<T*>(out), rows,
                                                       static_cast<int>(hidden / VEC));
    } else {
      const int grid = elementwise_grid(rows * hidden, 256);
      swiglu_fwd_scalar_kernel<T><<<grid, 256, 0, s>>>(static_cast<const T*>(gate_up),
                                                       static_cast<T*>(out), rows, hidden);
    }
  });
  return launch_status();
}

extern "C" int hlm_swiglu_bwd(const void* gate_up, const void* grad_out, void* grad_gate_up,
                              int64_t rows, int64_t hidden, int dtype, void* stream) {
  if (rows < 0 || hidden < 0) return HLM_ERR_INVALID_ARG;
  if (rows == 0 || hidden == 0) return HLM_OK;
  if (gate_up == nullptr || grad_out == nullptr || grad_gate_up == nullptr)
    return HLM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  LaunchScope scope(HLM_KERNEL_SWIGLU_BWD, s);
  HLM_DISPATCH_DTYPE(dtype, T, {
    constexpr int VEC = 16 / sizeof(T);
    const bool vec = (hidden % VEC == 0) && host_aligned16(gate_up) && host_aligned16(grad_out) &&
                     host_aligned16(grad_gate_up);
    if (vec && hidden / VEC <= (1ll << 30)) {
      constexpr int R = 2;
      const int grid = rows_grid(rows, R);
      swiglu_bwd_vec_kernel<T, R><<<grid, 256, 0, s>>>(
          static_cast<const T*>(gate_up), static_cast<const T*>(grad_out),
          static_cast<T*>(grad_gate_up), rows, static_cast<int>(hidden / VEC));
    } else {
      const int grid = elementwise_grid(rows * hidden, 256);
      swiglu_bwd_scalar_kernel<T><<<grid, 256, 0, s>>>(
          static_cast<const T*>(gate_up), static_cast<const T*>(grad_out),
          static_cast<T*>(grad_gate_up), rows, hidden);
    }
  });
  return launch_status();
}

extern "C" int hlm_residual_rms_norm_fwd(const void* residual, const void* branch,
                                         const void* weight, void* out, void* norm, int64_t rows,
                                         int64_t cols, float eps, int dtype, void* stream) {
  if (rows < 0 || cols < 0 || cols > (1ll << 30)) return HLM_ERR_INVALID_ARG;
  if (rows == 0 || cols == 0) return HLM_OK;
  if (branch == nullptr || norm == nullptr) return HLM_ERR_INVALID_ARG;
  if (residual != nullptr && out == nullptr) return HLM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int threads = 256, wpb = threads / 32;
  LaunchScope scope(HLM_KERNEL_RMSNORM_FWD, s);
  HLM_DISPATCH_DTYPE(dtype, T, {
    constexpr int VEC = 16 / sizeof(T);
    const int nv = pick_nv<T>(static_cast<int>(cols));
    const bool vec = nv > 0 && cols % VEC == 0 && host_aligned16(branch) && host_aligned16(norm) &&
                     (residual == nullptr || (host_aligned16(residual) && host_aligned16(out))) &&
                     (weight == nullptr || host_aligned16(weight));
    const int grid = rows_grid(rows, wpb);
    if (vec) {
      HLM_DISPATCH_NV(nv, NVC, {
        rmsnorm_fwd_vec_kernel<T, NVC><<<grid, threads, 0, s>>>(
            static_cast<const T*>(residual), static_cast<const T*>(branch),
            static_cast<const T*>(weight), static_cast<T*>(out), static_cast<T*>(norm), rows,
            static_cast<int>(cols), eps);
      });
    } else {
      rmsnorm_fwd_scalar_kernel<T><<<grid, threads, 0, s>>>(
          static_cast<const T*>(residual), static_cast<const T*>(branch),
          static_cast<const T*>(weight), static_cast<T*>(out), static_cast<T*>(norm), rows,
          static_cast<int>(cols), eps);
    }
  });
  return launch_status();
}

extern "C" size_t hlm_rms_norm_bwd_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return static_cast<size_t>(rms_bwd_weight_blocks(rows)) * kRmsBwdWarps *
         static_cast<size_t>(cols) * sizeof(float);
}

extern "C" int hlm_residual_rms_norm_bwd(const void* x, const void* weight, const void* grad_out,
                                         const void* grad_norm, void* grad_in, void* grad_weight,
                                         void* workspace, size_t workspace_bytes, int64_t rows,
                                         int64_t cols, float eps, int dtype, void* stream) {
  if (rows < 0 || cols < 0 || cols > (1ll << 30)) return HLM_ERR_INVALID_ARG;
  if (cols == 0) return HLM_OK;
  if (x == nullptr || grad_norm == nullptr || grad_in == nullptr) {
    if (rows != 0) return HLM_ERR_INVALID_ARG;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool want_w = weight != nullptr && grad_weight != nullptr;
  float* partial = nullptr;
  int grid = 1;
  const int threads = kRmsBwdThreads;
  if (want_w) {
    if (workspace == nullptr || workspace_bytes < hlm_rms_norm_bwd_workspace_bytes(rows, cols))
      return HLM_ERR_WORKSPACE;
    partial = static_cast<float*>(workspace);
    grid = rms_bwd_weight_blocks(rows);
  } else {
    grid = rows_grid(rows, kRmsBwdWarps);
  }
  HLM_DISPATCH_DTYPE(dtype, T, {
    if (rows > 0) {
      LaunchScope scope(HLM_KERNEL_RMSNORM_BWD, s);
      constexpr int VEC = 16 / sizeof(T);
      const int nv = pick_nv<T>(static_cast<int>(cols));
      const bool vec = nv > 0 && cols % VEC == 0 && host_aligned16(x) &&
                       host_aligned16(grad_norm) && host_aligned16(grad_in) &&
                       (grad_out == nullptr || host_aligned16(grad_out)) &&
                       (weight == nullptr || host_aligned16(weight));
      if (vec) {
        if (want_w) {
          HLM_DISPATCH_NV(nv, NVC, {
            rmsnorm_bwd_vec_kernel<T, NVC, true><<<grid, threads, 0, s>>>(
                static_cast<const T*>(x), static_cast<const T*>(weight),
                static_cast<const T*>(grad_out), static_cast<const T*>(grad_norm),
                static_cast<T*>(grad_in), partial, rows, static_cast<int>(cols), eps);
          });
        } else {
          HLM_DISPATCH_NV(nv, NVC, {
            rmsnorm_bwd_vec_kernel<T, NVC, false><<<grid, threads, 0, s>>>(
                static_cast<const T*>(x), nullptr, static_cast<const T*>(grad_out),
                static_cast<const T*>(grad_norm), static_cast<T*>(grad_in), nullptr, rows,
                static_cast<int>(cols), eps);
          });
        }
      } else {
        rmsnorm_bwd_scalar_kernel<T><<<grid, threads, 0, s>>>(
            static_cast<const T*>(x), static_cast<const T*>(weight),
            static_cast<const T*>(grad_out), static_cast<const T*>(grad_norm),
            static_cast<T*>(grad_in), partial, rows, static_cast<int>(cols), eps);
      }
    } else if (want_w) {
      // No rows: dweight is zero.
      if (cudaMemsetAsync(partial, 0, static_cast<size_t>(cols) * sizeof(float), s) !=
          cudaSuccess)
        return HLM_ERR_LAUNCH;
    }
    if (want_w) {
      const int nparts = rows > 0 ? grid * kRmsBwdWarps : 1;
      LaunchScope scope(0, s);
      reduce_partials_kernel<T><<<static_cast<int>((cols + 255) / 256), 256, 0, s>>>(
          partial, static_cast<T*>(grad_weight), nparts, static_cast<int>(cols));
    }
  });
  return launch_status();
}

extern "C" int hlm_scale_by_device_scalar(void* data, const float* scale, int64_t n, int dtype,
                                          void* stream) {
  if (n < 0) return HLM_ERR_INVALID_ARG;
  if (n == 0) return HLM_OK;
  if (data == nullptr || scale == nullptr) return HLM_ERR_INVALID_ARG;
  if (!host_aligned16(data)) return HLM_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  HLM_DISPATCH_DTYPE(dtype, T, {
    constexpr int VEC = 16 / sizeof(T);
    const int grid = elementwise_grid(n / VEC + 1, 256);
    LaunchScope scope(0, s);
    scale_kernel<T><<<grid, 256, 0, s>>>(static_cast<T*>(data), scale, n);
  });
  return launch_status();
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the weighted RMSNorm backward.
//
// Some callers cannot allocate device memory at the moment they need this
// operator: a host that pre-plans every device byte up front (a serving
// process with a fixed memory budget, or a framework whose allocator must
// account for all memory and cannot be re-entered from inside an operator),
// and code that must not stall the device, since cudaMalloc/cudaFree
// synchronise.  For them the dweight partial sums live in the fixed
// file-scope array below instead of a caller-provided workspace.  The array
// is sized for kNoAllocMaxCols columns (4 MiB) and every GPU that loads this
// library holds it until the process exits.
// ---------------------------------------------------------------------------
namespace hlm {

constexpr int kNoAllocMaxCols = HLM_NOALLOC_RMS_MAX_COLS;
constexpr int kNoAllocPartials = kRmsBwdMaxBlocks * kRmsBwdWarps;

static __device__ __align__(256) float g_noalloc_rms_partial[kNoAllocPartials * kNoAllocMaxCols];

// Device address of g_noalloc_rms_partial on the current device.  The
// host-side symbol is only a stand-in and must never be handed to a kernel.
// Outside stream capture the address is looked up again on every call (with
// the device current), so a context re-created after cudaDeviceReset gets the
// new address; inside a capture the lookup (which may load the module) is not
// allowed, so the address cached by an earlier uncaptured call on this device
// is used, and without one the call is refused with HLM_ERR_UNSUPPORTED.
static float* noalloc_partial_ptr(cudaStream_t stream, int* rc) {
  static float* ptrs[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *rc = HLM_ERR_LAUNCH;
    return nullptr;
  }
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess) {
    *rc = HLM_ERR_LAUNCH;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (capture == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_rms_partial) != cudaSuccess || p == nullptr) {
      *rc = HLM_ERR_LAUNCH;
      return nullptr;
    }
    ptrs[dev] = static_cast<float*>(p);
  } else if (ptrs[dev] == nullptr) {
    *rc = HLM_ERR_UNSUPPORTED;  // first call on this device made inside a stream capture
    return nullptr;
  }
  *rc = HLM_OK;
  return ptrs[dev];
}

}  // namespace hlm

extern "C" int hlm_residual_rms_norm_bwd_noalloc(const void* x, const void* weight,
                                                 const void* grad_out, const void* grad_norm,
                                                 void* grad_in, void* grad_weight, int64_t rows,
                                                 int64_t cols, float eps, int dtype,
                                                 void* stream) {
  if (rows < 0 || cols < 0) return HLM_ERR_INVALID_ARG;
  if (cols > kNoAllocMaxCols) return HLM_ERR_UNSUPPORTED;  // beyond the fixed scratch array
  if (weight == nullptr || grad_weight == nullptr) return HLM_ERR_INVALID_ARG;
  if (cols == 0) return HLM_OK;
  if (rows > 0 && (x == nullptr || grad_norm == nullptr || grad_in == nullptr))
    return HLM_ERR_INVALID_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = HLM_OK;
  float* partial = noalloc_partial_ptr(s, &rc);
  if (partial == nullptr) return rc;
  const int threads = kRmsBwdThreads;
  const int grid = rms_bwd_weight_blocks(rows);  // <= kRmsBwdMaxBlocks
  HLM_DISPATCH_DTYPE(dtype, T, {
    if (rows > 0) {
      // Every partial slot that the reduction below reads is written by this
      // launch first, so nothing left in the array by an earlier call is read.
      LaunchScope scope(HLM_KERNEL_RMSNORM_BWD, s);
      constexpr int VEC = 16 / sizeof(T);
      const int nv = pick_nv<T>(static_cast<int>(cols));
      const bool vec = nv > 0 && cols % VEC == 0 && host_aligned16(x) &&
                       host_aligned16(grad_norm) && host_aligned16(grad_in) &&
                       (grad_out == nullptr || host_aligned16(grad_out)) && host_aligned16(weight);
      if (vec) {
        HLM_DISPATCH_NV(nv, NVC, {
          rmsnorm_bwd_vec_kernel<T, NVC, true><<<grid, threads, 0, s>>>(
              static_cast<const T*>(x), static_cast<const T*>(weight),
              static_cast<const T*>(grad_out), static_cast<const T*>(grad_norm),
              static_cast<T*>(grad_in), partial, rows, static_cast<int>(cols), eps);
        });
      } else {
        rmsnorm_bwd_scalar_kernel<T><<<grid, threads, 0, s>>>(
            static_cast<const T*>(x), static_cast<const T*>(weight),
            static_cast<const T*>(grad_out), static_cast<const T*>(grad_norm),
            static_cast<T*>(grad_in), partial, rows, static_cast<int>(cols), eps);
      }
    } else {
      // No rows: dweight is zero; the one slot read below must start at zero.
      if (cudaMemsetAsync(partial, 0, static_cast<size_t>(cols) * sizeof(float), s) != cudaSuccess)
        return HLM_ERR_LAUNCH;
    }
    const int nparts = rows > 0 ? grid * kRmsBwdWarps : 1;
    LaunchScope scope(0, s);
    reduce_partials_kernel<T><<<static_cast<int>((cols + 255) / 256), 256, 0, s>>>(
        partial, static_cast<T*>(grad_weight), nparts, static_cast<int>(cols));
  });
  return launch_status();
}
