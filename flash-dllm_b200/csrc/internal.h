// Host-side helpers shared by the .cu translation units of the library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace fdllm {

// Device address of this process's status word on the current device
// (int32[4], see common.cuh::report).  nullptr if it cannot be resolved.
int32_t* status_ptr();

// Number of SMs of the current device (cached per device).
int sm_count();

// 2-D row-major bf16 tensor map with 128-byte swizzle: `rows` x `cols`
// elements, row pitch `ld` elements, box of `box_rows` x 64 elements.
// Returns FDLLM_OK or an error code.  Maps are cached by their arguments.
int make_tmap_bf16_sw128(CUtensorMap* out, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows);

// Integer tuning override from the environment; `dflt` if unset.
int env_int(const char* name, int dflt);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Programmatic dependent launch of the hot kernels on (FDLLM_PDL=0: off).
inline bool pdl_enabled() {
  static const bool on = env_int("FDLLM_PDL", 1) != 0;
  return on;
}

// Launch `kernel` with a cluster of `cluster_x` CTAs along x (> 1 only) and,
// when `pdl`, programmatic stream serialisation: the kernel may start while
// the previous kernel of the stream still runs and calls pdl_wait() before
// reading that kernel's results.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                             unsigned cluster_x, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  unsigned n = 0;
  if (cluster_x > 1) {
    attrs[n].id = cudaLaunchAttributeClusterDimension;
    attrs[n].val.clusterDim.x = cluster_x;
    attrs[n].val.clusterDim.y = 1;
    attrs[n].val.clusterDim.z = 1;
    ++n;
  }
  if (pdl) {
    attrs[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// QKV projection + RoPE + scatter through the stream-K GEMM (gemm_sk.cu) and
// its workspace size.
int launch_qkv_sk(const void* xn, const void* wq, const void* wk, const void* wv, const int64_t* pos,
                  const float* rope_sin, const float* rope_cos, void* q_out, void* k_out, void* v_out, int32_t n_rows,
                  int32_t d_model, int32_t n_heads, int64_t n_slots, void* workspace, size_t workspace_bytes,
                  int kv_by_slot, cudaStream_t stream);
size_t qkv_sk_ws_bytes(int32_t n_rows, int32_t d_model);

}  // namespace fdllm
