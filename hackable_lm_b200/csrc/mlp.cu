// gate_up projection with the SwiGLU activation in the GEMM epilogue: the
// reference's GateUpProjection.fwd_triton (model.py:291-292), i.e. a cuBLAS
// GEMM x @ W_gate_up^T followed by swiglu_triton (kernels.py:743-753), as one
// CTA-pair tcgen05 GEMM.
//
//   gate_up[M, 2H] = x[M, C] @ W[2H, C]^T   (bf16, kept for the backward)
//   h[M, H]        = silu(gate) * up        (fp32 math on the bf16-rounded
//                                            gate/up, like the reference)
//
// A pair tile covers 256 rows and 128 hidden units: CTA 0 loads the 128 gate
// rows of W and CTA 1 the matching 128 up rows (GemmParams::b_pair_stride = H),
// so every accumulator row holds [gate(128) | up(128)] and the epilogue can
// form h without another pass over gate_up.
#include "gemm_sm100.cuh"

namespace hlm {

// Four epilogue warps (one per TMEM lane quadrant, both 64-unit groups each)
// leave shared memory for five stages: measured 8% faster than eight warps
// (two per quadrant) with four stages at X [32768,768], W [4096,768].
constexpr int kMlpStages = 5;
constexpr int kMlpEpiWarps = 4;
constexpr int kMlpBwdStages = 3;  // 3 x 32 KB stages + 128 KB of epilogue boxes (two groups in flight per warp)

// Epilogue: per warp (32 rows) and 64-unit group: gate and up (2 x 64 fp32
// columns from TMEM) rounded to bf16 and staged as two 32x64 boxes for the
// gate_up output, h = silu(gate) * up staged as a third box; one lane issues
// the three TMA stores.
struct EpiSwiGLU {
  struct Params {
    alignas(64) CUtensorMap map_gu;  // gate_up [M][2H] bf16, box {64, 32}
    alignas(64) CUtensorMap map_h;   // h [M][H] bf16, box {64, 32}
    int H;
  };
  static constexpr int kBoxBytes = 32 * 128;
  template <int EPI_WARPS>
  static constexpr int smem_bytes() {
    return EPI_WARPS * 3 * kBoxBytes;
  }

  // Warp `part` of kParts (1 or 2) sharing a lane quadrant takes every
  // kParts-th 64-unit group; each group is processed in two 32-column halves
  // to keep the register footprint small.
  template <int BN, int kParts>
  static HLM_DEVICE void run(const Params& ep, const GemmParams& p, uint8_t* smem, uint32_t taddr,
                             int m_tile, int n_tile, int, int quad, int part, int lane) {
    static_assert(BN == 256 && (kParts == 1 || kParts == 2), "128 gate + 128 up columns");
    const uint32_t buf = smem_u32(smem) + static_cast<uint32_t>((part * 4 + quad) * 3 * kBoxBytes);
    const int row0 = m_tile * kBM + quad * 32;
#pragma unroll 1
    for (int g = part; g < 2; g += kParts) {
      // the stores that last used the staging boxes must have read them
      if (lane == 0) bulk_wait_group_read<0>();
      __syncwarp();
#pragma unroll 1
      for (int hs = 0; hs < 2; ++hs) {
        uint32_t pg[16], pu[16], ph[16];
        {
          uint32_t a[32], b[32];
          tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(g * 64 + hs * 32), a);
          tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(128 + g * 64 + hs * 32), b);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            pg[j] = pack_bf16x2(__uint_as_float(a[2 * j]), __uint_as_float(a[2 * j + 1]));
            pu[j] = pack_bf16x2(__uint_as_float(b[2 * j]), __uint_as_float(b[2 * j + 1]));
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float g0 = bf16_lo(pg[j]), g1 = bf16_hi(pg[j]);
          const float u0 = bf16_lo(pu[j]), u1 = bf16_hi(pu[j]);
          ph[j] = pack_bf16x2(g0 * sigmoid_fast(g0) * u0, g1 * sigmoid_fast(g1) * u1);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int cc = hs * 4 + c;  // 16-byte chunk of the 128-byte row
          const uint32_t off = static_cast<uint32_t>(lane * 128 + ((cc ^ (lane & 7)) << 4));
          st_shared_v4(buf + off, make_uint4(pg[4 * c], pg[4 * c + 1], pg[4 * c + 2], pg[4 * c + 3]));
          st_shared_v4(buf + kBoxBytes + off,
                       make_uint4(pu[4 * c], pu[4 * c + 1], pu[4 * c + 2], pu[4 * c + 3]));
          st_shared_v4(buf + 2 * kBoxBytes + off,
                       make_uint4(ph[4 * c], ph[4 * c + 1], ph[4 * c + 2], ph[4 * c + 3]));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 < p.M) {
        const int col = n_tile * 128 + g * 64;  // hidden unit of the group's first column
        tma_store_2d(&ep.map_gu, col, row0, buf);
        tma_store_2d(&ep.map_gu, ep.H + col, row0, buf + kBoxBytes);
        tma_store_2d(&ep.map_h, col, row0, buf + 2 * kBoxBytes);
        bulk_commit_group();
      }
    }
  }
};

// Backward of the MLP's SwiGLU fused into the down projection's grad_h GEMM:
//   grad_h[M, H]    = grad_y[M, C] @ W_down[C, H]        (rounded to bf16, as
//                                                         the reference's GEMM output)
//   grad_gate_up    = swiglu_backward(gate_up, grad_h)  (kernels.py:690-700,
//                                                         same fp32 arithmetic as
//                                                         swiglu_bwd_vec_kernel)
// grad_h never goes to memory.  Epilogue: 8 warps, two per TMEM lane quadrant
// (32 rows each), each taking every other 64-unit group of the 256-column
// tile.  A warp's gate and up boxes (32 x 64 bf16 each) of both its groups are
// loaded by TMA at the start of the tile into two 8 KB buffers (one mbarrier
// each), so the second group's load runs while the first is computed; dgate /
// dup are computed row by row and written back in place, and each buffer goes
// out with two TMA stores; a buffer's next load waits until those stores have
// read it.  (Two buffers per warp leave room for three mainloop stages; measured
// 143.7 us vs 151.5 us with one buffer and five stages at the d12 shape.)  The
// barrier phases continue across tiles through a per-warp tile counter kept in
// shared memory.
struct EpiSwiGLUBwd {
  struct Params {
    alignas(64) CUtensorMap map_gu;   // gate_up [M][2H] bf16, box {64, 32}
    alignas(64) CUtensorMap map_out;  // grad_gate_up [M][2H] bf16, box {64, 32}
    int H;
  };
  static constexpr int kBoxBytes = 32 * 128;
  static constexpr int kWarps = 8;
  static constexpr int kWarpBytes = 4 * kBoxBytes;  // per group: gate box, up box (outputs in place)
  static constexpr int kBarOffset = kWarps * kWarpBytes;
  static constexpr int kCtrOffset = kBarOffset + kWarps * 16;
  template <int EPI_WARPS>
  static constexpr int smem_bytes() {
    static_assert(EPI_WARPS == kWarps, "two epilogue warps per lane quadrant");
    return kCtrOffset + kWarps * 4;
  }
  static HLM_DEVICE void init(uint8_t* smem) {
    const uint32_t b = smem_u32(smem);
    for (int w = 0; w < 2 * kWarps; ++w) mbar_init(b + kBarOffset + 8 * w, 1);
    for (int w = 0; w < kWarps; ++w) {
      reinterpret_cast<volatile uint32_t*>(smem + kCtrOffset)[w] = 0u;
    }
  }

  template <int BN, int kParts>
  static HLM_DEVICE void run(const Params& ep, const GemmParams& p, uint8_t* smem, uint32_t taddr,
                             int m_tile, int n_tile, int, int quad, int part, int lane) {
    static_assert(BN == 256 && kParts == 2, "two warps per quadrant, two 64-unit groups each");
    const int row0 = m_tile * kBM + quad * 32;
    if (row0 >= p.M) return;  // no rows of this warp in the tile: no loads, barrier phase unchanged
    const int slot = part * 4 + quad;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t wbase = sbase + static_cast<uint32_t>(slot * kWarpBytes);
    volatile uint32_t* ctr = reinterpret_cast<volatile uint32_t*>(smem + kCtrOffset) + slot;
    const int h0 = n_tile * BN;  // hidden unit of the tile's first column
    uint32_t n = 0;
    if (lane == 0) n = *ctr;
    n = __shfl_sync(0xffffffffu, n, 0);
    // both groups' boxes in flight at once (buffer k for group part + 2k)
    if (lane == 0) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int g = part + 2 * k;
        const uint32_t gb = wbase + static_cast<uint32_t>(k * 2 * kBoxBytes);
        const uint32_t bar = sbase + static_cast<uint32_t>(kBarOffset + 16 * slot + 8 * k);
        // the store that last read this buffer (previous tile, group k) must be done with it
        if (k == 0) bulk_wait_group_read<1>(); else bulk_wait_group_read<0>();
        mbar_arrive_expect_tx(bar, 2 * kBoxBytes);
        tma_load_2d(gb, &ep.map_gu, h0 + g * 64, row0, bar);
        tma_load_2d(gb + kBoxBytes, &ep.map_gu, ep.H + h0 + g * 64, row0, bar);
      }
    }
#pragma unroll 1
    for (int k = 0; k < 2; ++k) {
      const int g = part + 2 * k;
      const uint32_t gate_box = wbase + static_cast<uint32_t>(k * 2 * kBoxBytes);
      const uint32_t up_box = gate_box + kBoxBytes;
      const uint32_t bar = sbase + static_cast<uint32_t>(kBarOffset + 16 * slot + 8 * k);
      if (!warp_wait(bar, n & 1u, p.err, kDevErrTimeoutEpiLoad, lane)) return;
#pragma unroll 1
      for (int hs = 0; hs < 2; ++hs) {
        uint32_t d[32];
        tmem_ld_32x32b_x32(taddr + static_cast<uint32_t>(g * 64 + hs * 32), d);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int cc = hs * 4 + c;  // 16-byte chunk of the row's 128 bytes
          const uint32_t off = static_cast<uint32_t>(lane * 128 + ((cc ^ (lane & 7)) << 4));
          const uint4 gr = ld_shared_v4(gate_box + off);
          const uint4 ur = ld_shared_v4(up_box + off);
          const uint32_t gw[4] = {gr.x, gr.y, gr.z, gr.w};
          const uint32_t uw[4] = {ur.x, ur.y, ur.z, ur.w};
          uint32_t og[4], ou[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            // grad_h rounded to bf16 first, like the reference's GEMM output
            const uint32_t dh = pack_bf16x2(__uint_as_float(d[8 * c + 2 * j]), __uint_as_float(d[8 * c + 2 * j + 1]));
            float rg[2], ru[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float gv = e ? bf16_hi(gw[j]) : bf16_lo(gw[j]);
              const float uv = e ? bf16_hi(uw[j]) : bf16_lo(uw[j]);
              const float dv = e ? bf16_hi(dh) : bf16_lo(dh);
              const float sg = sigmoid_fast(gv);
              const float silu = gv * sg;
              const float dsilu = sg * (1.0f + gv * (1.0f - sg));
              rg[e] = dv * uv * dsilu;
              ru[e] = dv * silu;
            }
            og[j] = pack_bf16x2(rg[0], rg[1]);
            ou[j] = pack_bf16x2(ru[0], ru[1]);
          }
          // in place: each thread rewrites only the chunks of its own row it just read
          st_shared_v4(gate_box + off, make_uint4(og[0], og[1], og[2], og[3]));
          st_shared_v4(up_box + off, make_uint4(ou[0], ou[1], ou[2], ou[3]));
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&ep.map_out, h0 + g * 64, row0, gate_box);
        tma_store_2d(&ep.map_out, ep.H + h0 + g * 64, row0, up_box);
        bulk_commit_group();
      }
    }
    if (lane == 0) *ctr = n + 1;
  }
};

}  // namespace hlm

using namespace hlm;

extern "C" int hlm_gate_up_swiglu_fwd(const void* x, const void* w_gate_up, void* gate_up_out,
                                      void* h_out, int64_t M, int64_t C, int64_t H, void* stream) {
  if (M < 0 || C <= 0 || H <= 0) return HLM_ERR_INVALID_ARG;
  if (M == 0) return HLM_OK;
  if (x == nullptr || w_gate_up == nullptr || gate_up_out == nullptr || h_out == nullptr)
    return HLM_ERR_INVALID_ARG;
  if (C % 64 != 0 || H % 128 != 0 || M > (1ll << 31) - 512 || 2 * H > (1ll << 30))
    return HLM_ERR_UNSUPPORTED;
  if (!host_aligned16(x) || !host_aligned16(w_gate_up) || !host_aligned16(gate_up_out) ||
      !host_aligned16(h_out))
    return HLM_ERR_UNSUPPORTED;
  CUtensorMap mx, mw;
  if (!encode_bf16_map(&mx, x, C, M, C, kBM)) return HLM_ERR_DRIVER;
  if (!encode_bf16_map(&mw, w_gate_up, C, 2 * H, C, 64)) return HLM_ERR_DRIVER;
  EpiSwiGLU::Params ep;
  if (!encode_bf16_map(&ep.map_gu, gate_up_out, 2 * H, M, 2 * H, 32) ||
      !encode_bf16_map(&ep.map_h, h_out, H, M, H, 32))
    return HLM_ERR_DRIVER;
  ep.H = static_cast<int>(H);
  GemmParams p;
  // N counted in hidden units: n_tiles = H / 128 tiles of [128 gate | 128 up]
  gemm_tiling_pair(p, static_cast<int>(M), static_cast<int>(2 * H), static_cast<int>(C), 256, 1);
  p.n_tiles = static_cast<int>(H / 128);
  p.b_pair_stride = static_cast<int>(H);
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  return launch_gemm_pair<256, kMlpStages, false, false, EpiSwiGLU, kMlpEpiWarps>(
      mx, mx, mx, mw, p, ep, static_cast<cudaStream_t>(stream), HLM_KERNEL_GATE_UP);
}

extern "C" int hlm_swiglu_down_bwd(const void* grad_y, const void* w_down, const void* gate_up,
                                   void* grad_gate_up, int64_t M, int64_t C, int64_t H, void* stream) {
  if (M < 0 || C <= 0 || H <= 0) return HLM_ERR_INVALID_ARG;
  if (M == 0) return HLM_OK;
  if (grad_y == nullptr || w_down == nullptr || gate_up == nullptr || grad_gate_up == nullptr)
    return HLM_ERR_INVALID_ARG;
  if (C % 64 != 0 || H % 256 != 0 || M > (1ll << 31) - 512 || 2 * H > (1ll << 30))
    return HLM_ERR_UNSUPPORTED;
  if (!host_aligned16(grad_y) || !host_aligned16(w_down) || !host_aligned16(gate_up) ||
      !host_aligned16(grad_gate_up))
    return HLM_ERR_UNSUPPORTED;
  CUtensorMap ma, mb;
  if (!encode_bf16_map(&ma, grad_y, C, M, C, kBM)) return HLM_ERR_DRIVER;  // A [M][C], K-major
  if (!encode_bf16_map(&mb, w_down, H, C, H, 64)) return HLM_ERR_DRIVER;   // B = W_down [C][H], N-major
  EpiSwiGLUBwd::Params ep;
  if (!encode_bf16_map(&ep.map_gu, gate_up, 2 * H, M, 2 * H, 32) ||
      !encode_bf16_map(&ep.map_out, grad_gate_up, 2 * H, M, 2 * H, 32))
    return HLM_ERR_DRIVER;
  ep.H = static_cast<int>(H);
  GemmParams p;
  gemm_tiling_pair(p, static_cast<int>(M), static_cast<int>(H), static_cast<int>(C), 256, 1);
  p.err = device_error_ptr();
  if (p.err == nullptr) return HLM_ERR_LAUNCH;
  return launch_gemm_pair<256, kMlpBwdStages, false, true, EpiSwiGLUBwd, EpiSwiGLUBwd::kWarps>(
      ma, ma, ma, mb, p, ep, static_cast<cudaStream_t>(stream), HLM_KERNEL_SWIGLU_DOWN_BWD);
}
