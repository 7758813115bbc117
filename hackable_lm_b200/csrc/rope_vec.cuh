// Vector QK-norm + RoPE kernels shared by the standalone op and the fused QKV
// backward (definitions in qk_norm_rope.cu).
#pragma once

#include "hlm_common.cuh"

namespace hlm {

enum RopeKernelMode : int { kRopeFwd = 0, kRopeBwdX = 1, kRopeBwdY = 2 };

struct RopeArgs {
  const void* xq;  // fwd/bwdX: inputs (strides qs); bwdY: saved outputs (strides qs)
  const void* xk;
  const void* gq;  // bwd: upstream gradients, contiguous [tokens][H][D]
  const void* gk;
  const float* rstd;  // bwdY: [tokens][Hq+Hk]
  const void* cosp;
  const void* sinp;
  void* oq;  // outputs, contiguous [tokens][H][D]
  void* ok;
  int64_t qs0, qs1, qs2, ks0, ks1, ks2, cs_stride;
  uint32_t tokens, T;
  int Hq, Hk, D, rd;
  float eps;
};

// Launch the vector kernel; HLM_ERR_UNSUPPORTED when the layout does not allow it.
template <typename T, int MODE>
int rope_vec_launch(const RopeArgs& a, int cs_dtype, int kernel_id, cudaStream_t s);

}  // namespace hlm
