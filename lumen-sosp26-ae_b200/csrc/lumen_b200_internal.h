// Declarations shared by the translation units of liblumen_b200.so.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/lumen_b200.h"
#include "sm100_ptx.cuh"

namespace b200 {

constexpr int kMaxExperts = 1024;  // bound of the per-expert tables kept in shared memory

// Number of SMs of the current device (cached per device).
int device_sm_count();

// Device address of the status word of the current device (cached per device);
// nullptr if the runtime refuses.  Kernels record the first wait that gave up there.
int* device_status_word();

// 2-D bf16 row-major tensor map with a {64 x box_rows} box and the 128-byte swizzle.
// `ld_elems` is the row pitch in elements (its byte size must be a multiple of 16).
// Returns 0 on success.
int encode_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols,
                        uint64_t ld_elems, uint32_t box_rows);

// 2-D row-major tensor map over bytes (fp8 codes) with a {128 x box_rows} box and the 128-byte
// swizzle; `ld_bytes` is the row pitch (a multiple of 16).  Returns 0 on success.
int encode_tmap_u8_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld_bytes,
                      uint32_t box_rows);

// General bf16 tensor map, rank <= 4, 128-byte swizzle; dims/strides innermost first,
// strides in bytes for dims 1..rank-1.
int encode_tmap_bf16(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides_bytes, const uint32_t* box);

}  // namespace b200
