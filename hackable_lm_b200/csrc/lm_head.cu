// Fused LM head + cross-entropy (forward and backward in one call), the B200
// restatement of _TritonFusedLinearCrossEntropy (kernels.py:878-942) and
// _linear_ce_kernel (kernels.py:291-318), with F.cross_entropy ignore_index
// semantics (ignored rows: no loss, no gradient; mean over the other rows).
//
// Per token chunk (the whole batch when it fits the logits budget):
//   1. logits GEMM   S = H_chunk @ W^T on tcgen05 (BN = 256 vocab columns per
//      tile); the epilogue rounds each logit to bf16 (the reference's logits
//      dtype), stores it, and folds it into a per-(row, tile) running
//      (max, sum exp) pair; the target logit is picked up in the tile that
//      holds it.  Full fp32 logits never exist in memory.
//   2. finalize      lse[row] = combine of the per-tile pairs; per-row loss;
//      deterministic per-block loss sums; per-row softmax data.
//   3. dlogits       in place: P = exp(S - lse) - onehot(target), zero for
//      ignored rows (the reference's in-place gradient overwrite,
//      kernels.py:315-318, without the 1/n factor)
//   4. dX GEMM       grad_hidden[chunk] = (P @ W) / n_valid     (W read N-major)
//   5. dW GEMM       grad_weight (+)= (P^T @ H_chunk) / n_valid (both MN-major)
// A pre-pass counts the valid targets of the whole batch so the 1/n_valid
// scale is known to every chunk on the device, with no host round trip.
// Within a chunk the dlogits passes of the later row parts run on a side stream,
// each alongside the grad_hidden GEMM of the part before it (see the chunk loop).
#include <mutex>

#include "gemm_sm100.cuh"

namespace hlm {

constexpr int kLmBN = 256;
constexpr int kLmPairStages = 6;  // CTA-pair logits GEMM (256 x 256 tiles)
constexpr int kLmBwdBN = 384;     // grad_hidden / grad_weight: 256 x 384 pair tiles (K = V or tokens)
constexpr int kLmBwdStages = 5;
constexpr int kLmEpiWarps = 8;
constexpr int kLmEpiParts = kLmEpiWarps / 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct LmStats {
  int n_valid;
  float inv_n;    // 1 / n_valid (0 when no row is valid)
  float loss_sum; // running sum of per-row losses over chunks
  int bad_target; // count of targets outside [0, V) that are not ignore_index
};

// Epilogue of the logits GEMM, run by 8 warps: two per TMEM lane quadrant,
// each taking every other 64-column group of the 256-column tile.  Per group:
// two tcgen05.ld (64 fp32), round to bf16 pairs (the reference's logits
// dtype), group max on the packed pairs, fold the rounded values into the
// row's running (max, sum 2^(x log2 e - max log2 e)), pick up the target logit
// in the group that holds it, and stage the bf16 group in a 128B-swizzled
// buffer (conflict-free 16-byte stores) that one lane writes to global memory
// with a TMA tensor store -- full 128-byte lines instead of per-thread
// partial-sector stores.
struct EpiLogitsLSE {
  struct Params {
    alignas(64) CUtensorMap store_map;  // logits [rows][V] bf16, box {64, 32}, 128B swizzle
    float2* partial;         // [n_tiles * parts][rows] (max, sum exp(x - max))
    float* tgt_logit;        // [rows]
    const int64_t* targets;  // [rows]
    int V;
    int rows;
  };
  static constexpr int kStageBytes = 32 * 128;  // one 32x64 bf16 box per warp
  template <int EPI_WARPS>
  static constexpr int smem_bytes() {
    return EPI_WARPS * kStageBytes;
  }

  template <int BN, int kParts>
  static HLM_DEVICE void run(const Params& ep, const GemmParams& p, uint8_t* smem, uint32_t taddr,
                             int m_tile, int n_tile, int, int quad, int part, int lane) {
    const int row = m_tile * kBM + quad * 32 + lane;
    const bool row_ok = row < p.M;
    const int n0 = n_tile * BN;
    // target column relative to this tile (-1: not in this tile)
    int trel = -1;
    if (row_ok) {
      const int64_t rel = ep.targets[row] - n0;
      if (rel >= 0 && rel < BN) trel = static_cast<int>(rel);
    }
    const uint32_t buf = smem_u32(smem) + static_cast<uint32_t>((part * 4 + quad) * kStageBytes);
    float m_run = -INFINITY, s_run = 0.0f;
#pragma unroll 1
    for (int g = part; g < BN / 64; g += kParts) {
      const int col0 = n0 + g * 64;
      uint32_t pk[32];
      {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(g * 64), r0);
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(g * 64 + 32), r1);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          pk[j] = pack_bf16x2(__uint_as_float(r0[2 * j]), __uint_as_float(r0[2 * j + 1]));
          pk[16 + j] = pack_bf16x2(__uint_as_float(r1[2 * j]), __uint_as_float(r1[2 * j + 1]));
        }
      }
      if (col0 + 64 > ep.V) {
        // ragged last group: columns at or past V (V is even) read as -inf
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + 2 * j >= ep.V) pk[j] = 0xff80ff80u;
      }
      // group max on the packed pairs (tree), then across the pair
      float gmax;
      {
        uint32_t t[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) t[j] = max_bf16x2(pk[j], pk[j + 16]);
#pragma unroll
        for (int w = 8; w > 0; w >>= 1)
#pragma unroll
          for (int j = 0; j < w; ++j) t[j] = max_bf16x2(t[j], t[j + w]);
        gmax = fmaxf(bf16_lo(t[0]), bf16_hi(t[0]));
      }
      const float new_m = fmaxf(m_run, gmax);
      if (new_m > -INFINITY) {
        const float nm2 = new_m * kLog2e;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          s0 += ex2_ftz(fmaf(bf16_lo(pk[j]), kLog2e, -nm2));
          s1 += ex2_ftz(fmaf(bf16_hi(pk[j]), kLog2e, -nm2));
          s2 += ex2_ftz(fmaf(bf16_lo(pk[j + 1]), kLog2e, -nm2));
          s3 += ex2_ftz(fmaf(bf16_hi(pk[j + 1]), kLog2e, -nm2));
        }
        s_run = s_run * ex2_ftz((m_run - new_m) * kLog2e) + ((s0 + s1) + (s2 + s3));
        m_run = new_m;
      }
      if (col0 < ep.V) {
        // the store that last used `buf` must have read it
        if (lane == 0) bulk_wait_group_read<0>();
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint32_t addr = buf + static_cast<uint32_t>(lane * 128 + ((c ^ (lane & 7)) << 4));
          st_shared_v4(addr, make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]));
        }
        // the target logit, read back from this thread's own staged row
        const int d = trel - g * 64;
        if (static_cast<unsigned>(d) < 64u) {
          const uint32_t addr = buf + static_cast<uint32_t>(lane * 128 + (((d >> 3) ^ (lane & 7)) << 4) +
                                                           (d & 7) * 2);
          uint16_t h;
          asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr) : "memory");
          ep.tgt_logit[row] = __uint_as_float(static_cast<uint32_t>(h) << 16);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          // the logits stream must not evict W (re-read by every row tile) from L2
          tma_store_2d_hint(&ep.store_map, col0, m_tile * kBM + quad * 32, buf, l2_policy_evict_first());
          bulk_commit_group();
        }
      }
    }
    if (row_ok)
      ep.partial[static_cast<int64_t>(n_tile * kParts + part) * ep.rows + row] =
          make_float2(m_run, s_run);
  }
};

__global__ void __launch_bounds__(1024) lm_count_valid_kernel(const int64_t* __restrict__ targets,
                                                             int64_t n, int64_t V,
                                                             int64_t ignore_index,
                                                             LmStats* __restrict__ stats) {
  __shared__ int s_valid[32], s_bad[32];
  int valid = 0, bad = 0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t t = targets[i];
    if (t == ignore_index) continue;
    if (t >= 0 && t < V)
      ++valid;
    else
      ++bad;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    valid += __shfl_xor_sync(0xffffffffu, valid, o);
    bad += __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if ((threadIdx.x & 31) == 0) {
    s_valid[threadIdx.x >> 5] = valid;
    s_bad[threadIdx.x >> 5] = bad;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int tv = 0, tb = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
      tv += s_valid[w];
      tb += s_bad[w];
    }
    stats->n_valid = tv;
    stats->inv_n = tv > 0 ? 1.0f / static_cast<float>(tv) : 0.0f;
    stats->loss_sum = 0.0f;
    stats->bad_target = tb;
  }
}

// Merge of two (max, sum 2^((x - max) log2 e)) pairs; empty pairs have sum 0.
HLM_DEVICE float2 lse_merge(float2 a, float2 b) {
  if (!(b.y > 0.0f)) return a;
  if (!(a.y > 0.0f)) return b;
  const float m = fmaxf(a.x, b.x);
  return make_float2(m, a.y * ex2_ftz((a.x - m) * kLog2e) + b.y * ex2_ftz((b.x - m) * kLog2e));
}

constexpr int kFinRows = 32;    // rows per block (one per lane)
constexpr int kFinGroups = 8;   // warps per block, each merging every 8th part

// Per row: lse from the per-(tile, part) pairs (row stride `stride`), the row
// loss, per-block loss sums, and the row's softmax data for the backward:
// {bits of lse*log2(e), target} for a valid row, {+inf, -1} for an ignored row
// (its gradient row is then exactly zero).  Warp g of a block merges parts
// g, g + 8, ... of the block's 32 rows (lane = row: 256-byte coalesced loads);
// the eight partial merges are combined in a fixed order.
__global__ void __launch_bounds__(kFinRows * kFinGroups) lm_finalize_kernel(
    const float2* __restrict__ partial, int n_parts, int stride, const float* __restrict__ tgt_logit,
    const int64_t* __restrict__ targets, int rows, int64_t V, int64_t ignore_index,
    int2* __restrict__ info_out, float* __restrict__ block_sums) {
  __shared__ float2 s_part[kFinGroups][kFinRows];
  const int lane = threadIdx.x & 31;
  const int g = threadIdx.x >> 5;
  const int row = blockIdx.x * kFinRows + lane;
  float2 acc = make_float2(-INFINITY, 0.0f);
  if (row < rows) {
    int t = g;
    for (; t + 3 * kFinGroups < n_parts; t += 4 * kFinGroups) {
      const float2 p0 = partial[static_cast<int64_t>(t) * stride + row];
      const float2 p1 = partial[static_cast<int64_t>(t + kFinGroups) * stride + row];
      const float2 p2 = partial[static_cast<int64_t>(t + 2 * kFinGroups) * stride + row];
      const float2 p3 = partial[static_cast<int64_t>(t + 3 * kFinGroups) * stride + row];
      acc = lse_merge(acc, lse_merge(lse_merge(p0, p1), lse_merge(p2, p3)));
    }
    for (; t < n_parts; t += kFinGroups) acc = lse_merge(acc, partial[static_cast<int64_t>(t) * stride + row]);
  }
  s_part[g][lane] = acc;
  __syncthreads();
  if (g == 0) {
    float loss = 0.0f;
    if (row < rows) {
      float2 m = s_part[0][lane];
#pragma unroll
      for (int k = 1; k < kFinGroups; ++k) m = lse_merge(m, s_part[k][lane]);
      const float lse = m.x + log2f(m.y) * kLn2;
      const int64_t t = targets[row];
      const bool valid = t != ignore_index && t >= 0 && t < V;
      if (valid) loss = lse - tgt_logit[row];
      info_out[row] = valid ? make_int2(__float_as_int(lse * kLog2e), static_cast<int>(t))
                            : make_int2(__float_as_int(INFINITY), -1);
    }
    loss = warp_sum(loss);
    if (lane == 0) block_sums[blockIdx.x] = loss;
  }
}

// Single block: add this chunk's block sums (fixed order) to the running sum;
// on the last chunk write loss = sum / n_valid.
__global__ void __launch_bounds__(256) lm_loss_reduce_kernel(const float* __restrict__ block_sums,
                                                            int n_blocks, LmStats* __restrict__ stats,
                                                            float* __restrict__ loss, int last) {
  __shared__ float s_sum[8];
  float v = 0.0f;
  for (int i = threadIdx.x; i < n_blocks; i += blockDim.x) v += block_sums[i];
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) s_sum[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = 0.0f;
    for (int w = 0; w < 8; ++w) b += s_sum[w];
    const float total = stats->loss_sum + b;
    stats->loss_sum = total;
    if (last) *loss = stats->n_valid > 0 ? total / static_cast<float>(stats->n_valid) : NAN;
  }
}


// In place: S -> P = softmax - onehot = 2^(S log2 e - lse log2 e) - [col == target],
// rounded to bf16 (the reference's in-place gradient overwrite,
// kernels.py:315-318); ignored rows carry lse log2 e = +inf and become zero.
// The 1/n_valid scale is applied in fp32 by the dX/dW GEMM epilogues: folded
// into the bf16 values it would carry one rounding error shared by every
// element.
// One block walks whole rows (the row's lse and target read once); each thread
// keeps kDlogitsU 16-byte loads in flight before it computes, since a single
// load per thread leaves too few bytes in flight to cover DRAM latency.
constexpr int kDlogitsU = 4;
__global__ void __launch_bounds__(256) lm_dlogits_kernel(__nv_bfloat16* __restrict__ logits,
                                                        const int2* __restrict__ info, int rows,
                                                        int64_t V) {
  const int vpr = static_cast<int>(V / 8);
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const int2 ri = info[row];
    const float nl2 = __int_as_float(ri.x);
    __nv_bfloat16* base = logits + static_cast<int64_t>(row) * V;
    for (int c0 = threadIdx.x; c0 < vpr; c0 += 256 * kDlogitsU) {
      uint4 x[kDlogitsU];
#pragma unroll
      for (int u = 0; u < kDlogitsU; ++u) {
        const int c = c0 + u * 256;
        if (c < vpr) x[u] = ld_global_v4(base + static_cast<int64_t>(c) * 8);
      }
#pragma unroll
      for (int u = 0; u < kDlogitsU; ++u) {
        const int c = c0 + u * 256;
        if (c >= vpr) break;
        const uint32_t xw[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
        float q[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          q[2 * e] = ex2_ftz(fmaf(bf16_lo(xw[e]), kLog2e, -nl2));
          q[2 * e + 1] = ex2_ftz(fmaf(bf16_hi(xw[e]), kLog2e, -nl2));
        }
        const int d = ri.y - c * 8;
        if (static_cast<unsigned>(d) < 8u) {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e == d) q[e] -= 1.0f;
        }
        st_global_v4(base + static_cast<int64_t>(c) * 8,
                     make_uint4(pack_bf16x2(q[0], q[1]), pack_bf16x2(q[2], q[3]), pack_bf16x2(q[4], q[5]),
                                pack_bf16x2(q[6], q[7])));
      }
    }
  }
}

__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float* __restrict__ src,
                                                         __nv_bfloat16* __restrict__ dst,
                                                         int64_t n) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

constexpr int kLmMaxParts = 4;  // row parts of a chunk's backward pipeline
static_assert(kLmMaxParts <= kSideEvents, "one side-stream event per part");

// ---------------------------------------------------------------------------
// Workspace plan
// ---------------------------------------------------------------------------
static constexpr int64_t kLogitsBudgetBytes = 4ll << 30;  // per-chunk bf16 logits

struct LmPlan {
  int64_t chunk;
  int n_chunks;
  int n_parts;
  size_t off_logits, off_partial, off_tgt, off_info, off_bsum, off_stats, off_dw, total;
};

static inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

static LmPlan lm_plan(int64_t n_tokens, int64_t C, int64_t V, int64_t chunk_tokens, bool want_dw) {
  LmPlan pl;
  int64_t chunk;
  if (chunk_tokens > 0) {
    chunk = ((chunk_tokens + kBM - 1) / kBM) * kBM;
  } else {
    chunk = kLogitsBudgetBytes / (V * 2);
    chunk = (chunk / kBM) * kBM;
    if (chunk < kBM) chunk = kBM;
  }
  if (chunk > n_tokens) chunk = n_tokens;
  if (chunk < 1) chunk = 1;
  pl.chunk = chunk;
  pl.n_chunks = static_cast<int>((n_tokens + chunk - 1) / chunk);
  pl.n_parts = static_cast<int>((V + kLmBN - 1) / kLmBN) * kLmEpiParts;
  size_t off = 0;
  pl.off_logits = off;
  off = align256(off + static_cast<size_t>(chunk) * V * 2);
  pl.off_partial = off;
  off = align256(off + static_cast<size_t>(pl.n_parts) * chunk * sizeof(float2));
  pl.off_tgt = off;
  off = align256(off + static_cast<size_t>(chunk) * 4);
  pl.off_info = off;
  off = align256(off + static_cast<size_t>(chunk) * 8);
  pl.off_bsum = off;
  off = align256(off + static_cast<size_t>((chunk + kFinRows - 1) / kFinRows) * 4);
  pl.off_stats = off;
  off = align256(off + sizeof(LmStats));
  pl.off_dw = off;
  if (want_dw && pl.n_chunks > 1) off = align256(off + static_cast<size_t>(V) * C * 4);
  pl.total = off;
  return pl;
}

}  // namespace hlm

using namespace hlm;

extern "C" size_t hlm_lm_head_ce_workspace_bytes(int64_t n_tokens, int64_t C, int64_t V,
                                                 int64_t chunk_tokens) {
  if (n_tokens <= 0 || C <= 0 || V <= 0) return 256;
  return lm_plan(n_tokens, C, V, chunk_tokens, true).total;
}

extern "C" int hlm_lm_head_ce(const void* hidden, const void* weight, const int64_t* targets,
                              float* loss, void* grad_hidden, void* grad_weight, void* workspace,
                              size_t workspace_bytes, int64_t n_tokens, int64_t C, int64_t V,
                              int64_t ignore_index, int64_t chunk_tokens, void* stream) {
  if (n_tokens <= 0 || C <= 0 || V <= 0) return HLM_ERR_INVALID_ARG;
  if (hidden == nullptr || weight == nullptr || targets == nullptr || loss == nullptr ||
      workspace == nullptr)
    return HLM_ERR_INVALID_ARG;
  if (C % 64 != 0 || V % 8 != 0) return HLM_ERR_UNSUPPORTED;
  if (n_tokens > (1ll << 30) || V > (1ll << 30) || C > 65536) return HLM_ERR_UNSUPPORTED;
  if (!host_aligned16(hidden) || !host_aligned16(weight) ||
      (grad_hidden != nullptr && !host_aligned16(grad_hidden)) ||
      (grad_weight != nullptr && !host_aligned16(grad_weight)))
    return HLM_ERR_UNSUPPORTED;
  const bool want_dx = grad_hidden != nullptr;
  const bool want_dw = grad_weight != nullptr;
  const LmPlan pl = lm_plan(n_tokens, C, V, chunk_tokens, want_dw);
  if (workspace_bytes < pl.total) return HLM_ERR_WORKSPACE;
  if (!host_aligned16(workspace)) return HLM_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* logits = reinterpret_cast<__nv_bfloat16*>(ws + pl.off_logits);
  float2* partial = reinterpret_cast<float2*>(ws + pl.off_partial);
  float* tgt_logit = reinterpret_cast<float*>(ws + pl.off_tgt);
  int2* info = reinterpret_cast<int2*>(ws + pl.off_info);
  float* bsum = reinterpret_cast<float*>(ws + pl.off_bsum);
  LmStats* stats = reinterpret_cast<LmStats*>(ws + pl.off_stats);
  float* dw_acc = reinterpret_cast<float*>(ws + pl.off_dw);
  int* err = device_error_ptr();
  if (err == nullptr) return HLM_ERR_LAUNCH;

  const __nv_bfloat16* H = static_cast<const __nv_bfloat16*>(hidden);
  const __nv_bfloat16* W = static_cast<const __nv_bfloat16*>(weight);

  {
    LaunchScope scope(0, s);
    lm_count_valid_kernel<<<1, 1024, 0, s>>>(targets, n_tokens, V, ignore_index, stats);
  }
  if (launch_status() != HLM_OK) return HLM_ERR_LAUNCH;

  // Tensor maps that do not depend on the chunk.
  CUtensorMap map_w_k, map_w_n;
  if (!encode_bf16_map(&map_w_k, W, C, V, C, 64)) return HLM_ERR_DRIVER;  // B boxes, logits GEMM
  if (!encode_bf16_map(&map_w_n, W, C, V, C, 64)) return HLM_ERR_DRIVER;     // B of dX GEMM

  for (int ci = 0; ci < pl.n_chunks; ++ci) {
    const int64_t r0 = static_cast<int64_t>(ci) * pl.chunk;
    const int rows = static_cast<int>(n_tokens - r0 < pl.chunk ? n_tokens - r0 : pl.chunk);
    const __nv_bfloat16* Hc = H + r0 * C;
    const int64_t* tc = targets + r0;
    const bool last = ci == pl.n_chunks - 1;

    // 1. logits + per-tile softmax statistics
    {
      CUtensorMap map_h;
      if (!encode_bf16_map(&map_h, Hc, C, rows, C, kBM)) return HLM_ERR_DRIVER;
      GemmParams p;
      gemm_tiling_pair(p, rows, static_cast<int>(V), static_cast<int>(C), kLmBN, 1);
      p.err = err;
      EpiLogitsLSE::Params ep;
      if (!encode_bf16_map(&ep.store_map, logits, V, rows, V, 32)) return HLM_ERR_DRIVER;
      ep.partial = partial;
      ep.tgt_logit = tgt_logit;
      ep.targets = tc;
      ep.V = static_cast<int>(V);
      ep.rows = rows;
      const int rc = launch_gemm_pair<kLmBN, kLmPairStages, false, false, EpiLogitsLSE, kLmEpiWarps>(
          map_h, map_h, map_h, map_w_k, p, ep, s, HLM_KERNEL_LM_LOGITS);
      if (rc != HLM_OK) return rc;
    }
    // 2. lse, per-row softmax data and loss
    {
      const int nb = (rows + kFinRows - 1) / kFinRows;
      {
        LaunchScope scope(0, s);
        lm_finalize_kernel<<<nb, kFinRows * kFinGroups, 0, s>>>(partial, pl.n_parts, rows, tgt_logit, tc,
                                                                 rows, V, ignore_index, info, bsum);
      }
      {
        LaunchScope scope(0, s);
        lm_loss_reduce_kernel<<<1, 256, 0, s>>>(bsum, nb, stats, loss, last ? 1 : 0);
      }
      if (launch_status() != HLM_OK) return HLM_ERR_LAUNCH;
    }
    const bool grads = want_dx || want_dw;
    if (!grads) continue;
    // 3. dlogits in place.  With grad_hidden wanted the rows split into up to
    // four parts (multiples of 256 rows, the pair tile, at least 1024 rows each);
    // part 0's pass runs alone on the caller's stream s, the others run one after
    // another on a side stream x, each beside the grad_hidden GEMM of the part
    // before it:
    //   s: dlogits(0) | dX(0)      | dX(1)      | dX(2)      | dX(3) dW
    //   x:            | dlogits(1) | dlogits(2) | dlogits(3) |
    // The GEMM keeps one CTA per SM busy on the tensor pipe and leaves issue
    // slots, registers and memory bandwidth that the streaming pass fills, so
    // only part 0's pass is exposed.  (Overlapping a pass with the logits GEMM
    // instead slows both: that GEMM's epilogue needs the issue slots and the
    // bandwidth itself.)
    int n_halves = 1;  // number of row parts
    int lo_of[kLmMaxParts] = {0}, hi_of[kLmMaxParts] = {rows};
    if (want_dx) {
      int parts = kLmMaxParts;
      while (parts > 1 && rows / parts < 1024) --parts;
      if (parts > 1) {
        const int step = ((rows / parts + 255) / 256) * 256;
        n_halves = 0;
        for (int r = 0; r < rows && n_halves < kLmMaxParts; r += step) {
          lo_of[n_halves] = r;
          hi_of[n_halves] = (n_halves == kLmMaxParts - 1 || r + step > rows) ? rows : r + step;
          if (hi_of[n_halves] == rows) {
            ++n_halves;
            break;
          }
          ++n_halves;
        }
      }
    }
    SideStream* side = nullptr;
    std::unique_lock<std::mutex> side_lock;
    if (n_halves > 1) {
      side = side_stream_of_current_device();
      if (side == nullptr) return HLM_ERR_LAUNCH;
      side_lock = std::unique_lock<std::mutex>(side->mu);
    }
    auto dlogits = [&](int r_lo, int r_hi, cudaStream_t st) -> int {
      const int n = r_hi - r_lo;
      if (n <= 0) return HLM_OK;
      int64_t blocks = n;  // whole rows per block
      const int64_t cap = static_cast<int64_t>(num_sms_of_current_device()) * 8;
      if (blocks > cap) blocks = cap;
      LaunchScope scope(HLM_KERNEL_LM_DLOGITS, st);
      lm_dlogits_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(logits + static_cast<int64_t>(r_lo) * V,
                                                                 info + r_lo, n, V);
      return launch_status();
    };
    {
      int rc = dlogits(lo_of[0], hi_of[0], s);
      if (rc != HLM_OK) return rc;
      if (n_halves > 1) {
        if (cudaEventRecord(side->ev_start, s) != cudaSuccess ||
            cudaStreamWaitEvent(side->stream, side->ev_start, 0) != cudaSuccess)
          return HLM_ERR_LAUNCH;
        for (int q = 1; q < n_halves; ++q) {
          rc = dlogits(lo_of[q], hi_of[q], side->stream);
          if (rc != HLM_OK) return rc;
          if (cudaEventRecord(side->ev_done[q], side->stream) != cudaSuccess) return HLM_ERR_LAUNCH;
        }
      }
    }
    // 4. grad_hidden[chunk] = P @ W, per half once its dlogits pass is done
    auto grad_hidden_gemm = [&](int r_lo, int r_hi) -> int {
      const int n = r_hi - r_lo;
      if (n <= 0) return HLM_OK;
      CUtensorMap map_p;
      if (!encode_bf16_map(&map_p, logits + static_cast<int64_t>(r_lo) * V, V, n, V, kBM))
        return HLM_ERR_DRIVER;
      GemmParams p;
      gemm_tiling_pair(p, n, static_cast<int>(C), static_cast<int>(V), kLmBwdBN, 1);
      p.err = err;
      EpiStore::Params ep;
      ep.d = static_cast<__nv_bfloat16*>(grad_hidden) + (r0 + r_lo) * C;
      ep.ldd = C;
      ep.split_stride = 0;
      ep.dtype = HLM_BF16;
      ep.accumulate = 0;
      ep.vec_ok = 1;
      ep.alpha = &stats->inv_n;
      return launch_gemm_pair<kLmBwdBN, kLmBwdStages, false, true, EpiStore>(
          map_p, map_p, map_p, map_w_n, p, ep, s, HLM_KERNEL_LM_DX);
    };
    for (int h = 0; h < n_halves; ++h) {
      // part h's rows are ready once the side stream's pass over them is done
      if (h > 0 && cudaStreamWaitEvent(s, side->ev_done[h], 0) != cudaSuccess) return HLM_ERR_LAUNCH;
      if (want_dx) {
        const int rc = grad_hidden_gemm(lo_of[h], hi_of[h]);
        if (rc != HLM_OK) return rc;
      }
    }
    // 5. grad_weight (+)= P^T @ H_chunk
    if (want_dw) {
      CUtensorMap map_pt, map_hn;
      if (!encode_bf16_map(&map_pt, logits, V, rows, V, 64)) return HLM_ERR_DRIVER;
      if (!encode_bf16_map(&map_hn, Hc, C, rows, C, 64)) return HLM_ERR_DRIVER;
      GemmParams p;
      gemm_tiling_pair(p, static_cast<int>(V), static_cast<int>(C), rows, kLmBwdBN, 1);
      p.err = err;
      EpiStore::Params ep;
      ep.ldd = C;
      ep.split_stride = 0;
      ep.vec_ok = 1;
      ep.alpha = &stats->inv_n;
      if (pl.n_chunks == 1) {
        ep.d = grad_weight;
        ep.dtype = HLM_BF16;
        ep.accumulate = 0;
      } else {
        ep.d = dw_acc;
        ep.dtype = HLM_F32;
        ep.accumulate = ci > 0 ? 1 : 0;
      }
      const int rc = launch_gemm_pair<kLmBwdBN, kLmBwdStages, true, true, EpiStore>(
          map_pt, map_pt, map_pt, map_hn, p, ep, s, HLM_KERNEL_LM_DW);
      if (rc != HLM_OK) return rc;
    }
  }
  if (want_dw && pl.n_chunks > 1) {
    const int64_t n = V * C;
    int64_t blocks = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(num_sms_of_current_device()) * 8;
    if (blocks > cap) blocks = cap;
    LaunchScope scope(0, s);
    f32_to_bf16_kernel<<<static_cast<int>(blocks), 256, 0, s>>>(
        dw_acc, static_cast<__nv_bfloat16*>(grad_weight), n);
    if (launch_status() != HLM_OK) return HLM_ERR_LAUNCH;
  }
  return HLM_OK;
}
