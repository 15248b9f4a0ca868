// RMSNorm with the reference's rounding points:
//   h = bf16( w * bf16( y * rsqrt(mean(y^2) + eps) ) )
// (RMSLayerNorm.forward in llada/model/modeling_llada.py:389-403: fp32
// normalise, cast to the input dtype, then the bf16 weight product), either
// of the input itself (y = x) or fused with the residual add before it,
// y = bf16(x + r) -- the `x = x + dropout(att); ff_norm(x)` pair of
// llada/flash_cache_triton.py:618-627 -- in which case y is written too.
//
// One CTA of kNormThreads per row: every thread issues all of its 16-byte
// loads (up to kNormMaxVec per input) before the block reduction, so each SM
// keeps several KB of loads in flight; the row stays in registers for the
// second (scaling) pass.
//
// SwiGLU: out = bf16(silu(gate)) * up with silu in fp32 and the product
// rounded to bf16, i.e. torch's `act(x) * x_up` on bf16 tensors
// (llada/flash_cache_triton.py:628-633).  gate and up may be the two column
// halves of one [rows, 2*cols] GEMM output; a 2-D grid (row, column chunk)
// avoids per-element index division.
#include "common.cuh"
#include "internal.h"

#include <algorithm>

namespace fdllm {

constexpr int kNormThreads = 128;
constexpr int kNormMaxVec = 8;  // 16-byte vectors per thread -> rows up to 128 * 8 * 8 = 8192 wide

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
  return t;
}

template <bool kAdd>
__global__ void __launch_bounds__(kNormThreads) norm_rows_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 const __nv_bfloat16* __restrict__ r,
                                                                 const __nv_bfloat16* __restrict__ w,
                                                                 __nv_bfloat16* __restrict__ y,
                                                                 __nv_bfloat16* __restrict__ h, int dim, float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_launch_dependents();  // the QKV GEMM may set up while the rows are normalised
  const int64_t base = static_cast<int64_t>(blockIdx.x) * dim;
  const uint4* xr = reinterpret_cast<const uint4*>(x + base);
  const uint4* rr = reinterpret_cast<const uint4*>(r + base);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  const int nvec = dim / 8;
  uint4 v[kNormMaxVec];
  uint4 b[kNormMaxVec];
#pragma unroll
  for (int k = 0; k < kNormMaxVec; ++k) {
    const int i = threadIdx.x + kNormThreads * k;
    if (i < nvec) {
      v[k] = xr[i];
      if (kAdd) b[k] = rr[i];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kNormMaxVec; ++k) {
    const int i = threadIdx.x + kNormThreads * k;
    if (i < nvec) {
      uint32_t* pv = reinterpret_cast<uint32_t*>(&v[k]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pv[j]));
        if (kAdd) {
          const float2 fb = __bfloat1622float2(reinterpret_cast<const __nv_bfloat162*>(&b[k])[j]);
          pv[j] = pack_bf16x2(f.x + fb.x, f.y + fb.y);
          f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&pv[j]));
        }
        ss += f.x * f.x + f.y * f.y;
      }
      if (kAdd) reinterpret_cast<uint4*>(y + base)[i] = v[k];
    }
  }
  const float rstd = rsqrtf(block_sum(ss, red) / static_cast<float>(dim) + eps);
  uint4* hr = reinterpret_cast<uint4*>(h + base);
#pragma unroll
  for (int k = 0; k < kNormMaxVec; ++k) {
    const int i = threadIdx.x + kNormThreads * k;
    if (i < nvec) {
      const uint4 wv = wr[i];
      const __nv_bfloat162* ps = reinterpret_cast<const __nv_bfloat162*>(&v[k]);
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

constexpr int kSwigluThreads = 256;
constexpr int kSwigluVec = 2;  // 16-byte vectors per thread

__global__ void __launch_bounds__(kSwigluThreads) swiglu_kernel(const __nv_bfloat16* __restrict__ g,
                                                                const __nv_bfloat16* __restrict__ u,
                                                                __nv_bfloat16* __restrict__ out, int cols_vec,
                                                                int64_t ld_in) {
  const int64_t row = blockIdx.y;
  const uint4* gr = reinterpret_cast<const uint4*>(g + row * ld_in);
  const uint4* ur = reinterpret_cast<const uint4*>(u + row * ld_in);
  uint4* orow = reinterpret_cast<uint4*>(out) + row * cols_vec;
  const int c0 = blockIdx.x * (kSwigluThreads * kSwigluVec) + threadIdx.x;
  uint4 a[kSwigluVec], b[kSwigluVec];
#pragma unroll
  for (int k = 0; k < kSwigluVec; ++k) {
    const int c = c0 + k * kSwigluThreads;
    if (c < cols_vec) {
      a[k] = gr[c];
      b[k] = ur[c];
    }
  }
#pragma unroll
  for (int k = 0; k < kSwigluVec; ++k) {
    const int c = c0 + k * kSwigluThreads;
    if (c < cols_vec) {
      const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&a[k]);
      const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&b[k]);
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
      orow[c] = o;
    }
  }
}

bool norm_dim_ok(int32_t dim) { return dim > 0 && dim % 8 == 0 && dim / 8 <= kNormThreads * kNormMaxVec; }

}  // namespace fdllm

extern "C" int fdllm_rmsnorm(const void* x, const void* weight, void* y, int32_t rows, int32_t dim, float eps,
                             cudaStream_t stream) {
  if (rows < 0 || !fdllm::norm_dim_ok(dim)) return FDLLM_ERR_ARG;
  if (rows == 0) return FDLLM_OK;
  if (!x || !weight || !y || !fdllm::aligned16(x) || !fdllm::aligned16(weight) || !fdllm::aligned16(y))
    return FDLLM_ERR_ARG;
  fdllm::norm_rows_kernel<false><<<rows, fdllm::kNormThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), nullptr, static_cast<const __nv_bfloat16*>(weight), nullptr,
      static_cast<__nv_bfloat16*>(y), dim, eps);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

extern "C" int fdllm_add_rmsnorm(const void* x, const void* residual, const void* weight, void* y, void* h,
                                 int32_t rows, int32_t dim, float eps, cudaStream_t stream) {
  if (rows < 0 || !fdllm::norm_dim_ok(dim)) return FDLLM_ERR_ARG;
  if (rows == 0) return FDLLM_OK;
  const void* ptrs[] = {x, residual, weight, y, h};
  for (const void* p : ptrs)
    if (p == nullptr || !fdllm::aligned16(p)) return FDLLM_ERR_ARG;
  fdllm::norm_rows_kernel<true><<<rows, fdllm::kNormThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual),
      static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(y), static_cast<__nv_bfloat16*>(h), dim,
      eps);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}

extern "C" int fdllm_swiglu(const void* gate, const void* up, void* out, int64_t rows, int32_t cols,
                            int64_t ld_in, cudaStream_t stream) {
  if (rows < 0 || rows > 65535 || cols <= 0 || cols % 8 != 0 || ld_in < cols || ld_in % 8 != 0)
    return FDLLM_ERR_ARG;
  if (rows == 0) return FDLLM_OK;
  if (!gate || !up || !out || !fdllm::aligned16(gate) || !fdllm::aligned16(up) || !fdllm::aligned16(out))
    return FDLLM_ERR_ARG;
  const int cols_vec = cols / 8;
  const int per_cta = fdllm::kSwigluThreads * fdllm::kSwigluVec;
  const dim3 grid((cols_vec + per_cta - 1) / per_cta, static_cast<unsigned>(rows));
  fdllm::swiglu_kernel<<<grid, fdllm::kSwigluThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(gate),
                                                                   static_cast<const __nv_bfloat16*>(up),
                                                                   static_cast<__nv_bfloat16*>(out), cols_vec, ld_in);
  return cudaPeekAtLastError() == cudaSuccess ? FDLLM_OK : FDLLM_ERR_CUDA;
}
