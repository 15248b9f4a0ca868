// RMSNorm with the reference's rounding points:
//   y = bf16( w * bf16( x * rsqrt(mean(x^2) + eps) ) )
// (RMSLayerNorm.forward in llada/model/modeling_llada.py:389-403: fp32
// normalise, cast to the input dtype, then the bf16 weight product).
// One CTA per row, 16-byte vector loads.
#include "common.cuh"
#include "internal.h"

namespace fdllm {

constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               __nv_bfloat16* __restrict__ y, int dim, float eps) {
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * dim);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * dim);
  const int nvec = dim / 8;
  float ss = 0.f;
  for (int i = threadIdx.x; i < nvec; i += kNormThreads) {
    const uint4 v = xr[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      ss += f.x * f.x + f.y * f.y;
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float rstd = rsqrtf(red[0] / static_cast<float>(dim) + eps);
  for (int i = threadIdx.x; i < nvec; i += kNormThreads) {
    const uint4 v = xr[i];
    const uint4 wv = wr[i];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&wv);
    uint4 o;
    uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      const float2 gw = __bfloat1622float2(g[j]);
      const float2 n = __bfloat1622float2(__floats2bfloat162_rn(f.x * rstd, f.y * rstd));
      op[j] = pack_bf16x2(gw.x * n.x, gw.y * n.y);
    }
    yr[i] = o;
  }
}

}  // namespace fdllm

extern "C" int fdllm_rmsnorm(const void* x, const void* weight, void* y, int32_t rows, int32_t dim, float eps,
                             cudaStream_t stream) {
  if (rows < 0 || dim <= 0 || dim % 8 != 0) return FDLLM_ERR_ARG;
  if (rows == 0) return FDLLM_OK;
  if (!x || !weight || !y || !fdllm::aligned16(x) || !fdllm::aligned16(weight) || !fdllm::aligned16(y))
    return FDLLM_ERR_ARG;
  fdllm::rmsnorm_kernel<<<rows, fdllm::kNormThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(weight),
      static_cast<__nv_bfloat16*>(y), dim, eps);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}
