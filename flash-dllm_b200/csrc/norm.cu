// RMSNorm with the reference's rounding points:
//   y = bf16( w * bf16( x * rsqrt(mean(x^2) + eps) ) )
// (RMSLayerNorm.forward in llada/model/modeling_llada.py:389-403: fp32
// normalise, cast to the input dtype, then the bf16 weight product).
// One CTA per row, 16-byte vector loads.
#include "common.cuh"
#include "internal.h"

#include <algorithm>

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

// ---------------------------------------------------------------------------
// Residual add fused with the following RMSNorm, and the SwiGLU product.
//   y = x + r (bf16 rounding, like the reference's `x + att`), h = RMSNorm(y)
//   (modeling_llada.py:389-403 rounding points) -- flash_cache_triton.py:619-627.
//   out = bf16(silu(g)) * u with silu in fp32 and the product rounded to bf16,
//   i.e. torch's `act(x) * x_up` on bf16 tensors -- flash_cache_triton.py:628-633.
// One warp per row for the norm (4 rows per CTA, 16-byte vectors, two passes
// over a row held in registers up to 4096 wide); grid-stride for SwiGLU, whose
// gate and up may be the two column halves of one [rows, 2*cols] GEMM output.
// ---------------------------------------------------------------------------
namespace fdllm {

constexpr int kAddNormRows = 4;  // rows (warps) per CTA
constexpr int kAddNormMaxVec = 16;  // 16 x 8 bf16 per lane -> rows up to 4096

__global__ void __launch_bounds__(32 * kAddNormRows) add_rmsnorm_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ r, const __nv_bfloat16* __restrict__ w,
    __nv_bfloat16* __restrict__ y, __nv_bfloat16* __restrict__ h, int rows, int dim, float eps) {
  const int row = blockIdx.x * kAddNormRows + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = dim / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(row) * dim);
  const uint4* rr = reinterpret_cast<const uint4*>(r + static_cast<int64_t>(row) * dim);
  uint4* yr = reinterpret_cast<uint4*>(y + static_cast<int64_t>(row) * dim);
  uint4* hr = reinterpret_cast<uint4*>(h + static_cast<int64_t>(row) * dim);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4 sum[kAddNormMaxVec];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kAddNormMaxVec; ++k) {
    const int i = lane + 32 * k;
    if (i < nvec) {
      const uint4 a = xr[i], b = rr[i];
      const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
      const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
      uint32_t* po = reinterpret_cast<uint32_t*>(&sum[k]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = __bfloat1622float2(pa[j]), fb = __bfloat1622float2(pb[j]);
        po[j] = pack_bf16x2(fa.x + fb.x, fa.y + fb.y);
        const float2 s = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&po[j]));
        ss += s.x * s.x + s.y * s.y;
      }
      yr[i] = sum[k];
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / static_cast<float>(dim) + eps);
#pragma unroll
  for (int k = 0; k < kAddNormMaxVec; ++k) {
    const int i = lane + 32 * k;
    if (i < nvec) {
      const uint4 wv = wr[i];
      const __nv_bfloat162* ps = reinterpret_cast<const __nv_bfloat162*>(&sum[k]);
      const __nv_bfloat162* pw = reinterpret_cast<const __nv_bfloat162*>(&wv);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(ps[j]);
        const float2 g = __bfloat1622float2(pw[j]);
        const float2 n = __bfloat1622float2(__floats2bfloat162_rn(f.x * rstd, f.y * rstd));
        po[j] = pack_bf16x2(g.x * n.x, g.y * n.y);
      }
      hr[i] = o;
    }
  }
}

__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ g, const __nv_bfloat16* __restrict__ u,
                              __nv_bfloat16* __restrict__ out, int64_t rows, int cols_vec, int64_t ld_in) {
  const int64_t n_vec = rows * cols_vec;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_vec;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / cols_vec;
    const int64_t in = row * ld_in + 8 * (i - row * cols_vec);  // element offset of this vector's input
    const uint4 a = *reinterpret_cast<const uint4*>(g + in);
    const uint4 b = *reinterpret_cast<const uint4*>(u + in);
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fa = __bfloat1622float2(pa[j]), fb = __bfloat1622float2(pb[j]);
      // silu(a) = a / (1 + exp(-a)), rounded to bf16 before the product
      const float2 s = __bfloat1622float2(__floats2bfloat162_rn(fa.x / (1.f + expf(-fa.x)),
                                                                  fa.y / (1.f + expf(-fa.y))));
      po[j] = pack_bf16x2(s.x * fb.x, s.y * fb.y);
    }
    reinterpret_cast<uint4*>(out)[i] = o;
  }
}

}  // namespace fdllm

extern "C" int fdllm_add_rmsnorm(const void* x, const void* residual, const void* weight, void* y, void* h,
                                 int32_t rows, int32_t dim, float eps, cudaStream_t stream) {
  if (rows < 0 || dim <= 0 || dim % 8 != 0 || dim / 8 > 32 * fdllm::kAddNormMaxVec) return FDLLM_ERR_ARG;
  if (rows == 0) return FDLLM_OK;
  const void* ptrs[] = {x, residual, weight, y, h};
  for (const void* p : ptrs)
    if (p == nullptr || !fdllm::aligned16(p)) return FDLLM_ERR_ARG;
  const int grid = (rows + fdllm::kAddNormRows - 1) / fdllm::kAddNormRows;
  fdllm::add_rmsnorm_kernel<<<grid, 32 * fdllm::kAddNormRows, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual),
      static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(y), static_cast<__nv_bfloat16*>(h),
      rows, dim, eps);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

extern "C" int fdllm_swiglu(const void* gate, const void* up, void* out, int64_t rows, int32_t cols,
                            int64_t ld_in, cudaStream_t stream) {
  if (rows < 0 || cols <= 0 || cols % 8 != 0 || ld_in < cols || ld_in % 8 != 0) return FDLLM_ERR_ARG;
  if (rows == 0) return FDLLM_OK;
  if (!gate || !up || !out || !fdllm::aligned16(gate) || !fdllm::aligned16(up) || !fdllm::aligned16(out))
    return FDLLM_ERR_ARG;
  const int64_t n_vec = rows * (cols / 8);
  const int grid = static_cast<int>(std::min<int64_t>((n_vec + 255) / 256, 8 * fdllm::sm_count()));
  fdllm::swiglu_kernel<<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(gate),
                                                  static_cast<const __nv_bfloat16*>(up),
                                                  static_cast<__nv_bfloat16*>(out), rows, cols / 8, ld_in);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}
