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

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace fdllm
