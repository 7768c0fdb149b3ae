// Host-side helpers shared by the kernel launchers: TMA tensor-map encoding
// (through the driver entry point, so the library needs no -lcuda) and the
// per-device dynamic shared-memory opt-in.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

// 2-D map over a row-major [outer, inner] array whose rows are
// `row_stride_elems` elements apart; box = [box_outer, box_inner].
bool gl_make_tmap_2d(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, int64_t inner,
                     int64_t outer, int64_t row_stride_elems, uint32_t box_inner,
                     uint32_t box_outer, CUtensorMapSwizzle sw, const char** why);

// 3-D map: dims {d0 (innermost), d1, d2}, strides (in elements) of d1 and d2,
// box {b0, b1, b2}.
bool gl_make_tmap_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* ptr, int64_t d0,
                     int64_t d1, int64_t d2, int64_t s1_elems, int64_t s2_elems, uint32_t b0,
                     uint32_t b1, uint32_t b2, CUtensorMapSwizzle sw, const char** why);

// Raises the dynamic shared-memory limit of `func` on the current device
// (once per device and function).
bool gl_set_smem_attr(const void* func, int unused, int bytes, const char** why);
