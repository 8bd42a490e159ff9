// host_common.h — host-side helpers shared by the C-ABI entry points:
// TMA tensor-map encoding (driver entry point fetched through the runtime, so
// the library does not link libcuda), SM count, and status codes.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "../../include/nl_ops.h"

namespace nl {

inline PFN_cuTensorMapEncodeTiled_v12000 encode_tiled_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Row-major bf16 matrix [rows, cols] with row pitch `ld` elements, tiled as
// boxes of box_cols x box_rows with 128-byte swizzle (box_cols * 2 == 128).
inline int make_tmap_bf16_2d(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t ld,
                             uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_tiled_fn();
  if (!fn) return NL_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15)) return NL_ERR_ALIGN;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NL_OK : NL_ERR_CUDA;
}

// Output tile map for the GEMM epilogue's TMA stores: row-major [rows, cols]
// of f32 (128-byte swizzle) or bf16 (64-byte swizzle), boxes of 32 x 32.
inline int make_tmap_out_2d(CUtensorMap* m, const void* base, bool bf16, uint64_t cols, uint64_t rows,
                            uint64_t ld) {
  auto fn = encode_tiled_fn();
  if (!fn) return NL_ERR_CUDA;
  const uint64_t es = bf16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * es) & 15)) return NL_ERR_ALIGN;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * es};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  bf16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NL_OK : NL_ERR_CUDA;
}

// Batched row-major bf16 tensor [batch, rows, cols] (contiguous), boxes of
// box_cols x box_rows x 1 with 128-byte swizzle.  Rows past `rows` of one
// batch entry read as zero instead of spilling into the next entry.
inline int make_tmap_bf16_3d(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint64_t batch,
                             uint32_t box_cols, uint32_t box_rows) {
  auto fn = encode_tiled_fn();
  if (!fn) return NL_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((cols * 2) & 15)) return NL_ERR_ALIGN;
  cuuint64_t dims[3] = {cols, rows, batch};
  cuuint64_t strides[2] = {cols * 2, cols * rows * 2};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NL_OK : NL_ERR_CUDA;
}

// Strided 4-D bf16 tensor [b][h][s][64 cols] addressed with element strides
// (s_stride, h_stride, b_stride), boxes of 64 x box_rows x 1 x 1, SW128.
// Covers both contiguous [n, s, 64] (h = 1) and head-interleaved activations
// such as a fused QKV projection [b, s, 3, H, 64].
inline int make_tmap_bf16_4d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t heads, uint64_t batch,
                             uint64_t s_stride, uint64_t h_stride, uint64_t b_stride, uint32_t box_rows) {
  auto fn = encode_tiled_fn();
  if (!fn) return NL_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((s_stride * 2) & 15) || ((h_stride * 2) & 15) ||
      ((b_stride * 2) & 15))
    return NL_ERR_ALIGN;
  cuuint64_t dims[4] = {64, rows, heads, batch};
  cuuint64_t strides[3] = {s_stride * 2, h_stride * 2, b_stride * 2};
  cuuint32_t box[4] = {64, box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NL_OK : NL_ERR_CUDA;
}

// f32 [n, rows, 64] (contiguous) written by 32 x 32 boxes with 128-byte
// swizzle (one row of a box = 128 B); rows past `rows` are clipped per n.
inline int make_tmap_f32_rows64_3d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t n) {
  auto fn = encode_tiled_fn();
  if (!fn) return NL_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return NL_ERR_ALIGN;
  cuuint64_t dims[3] = {64, rows, n};
  cuuint64_t strides[2] = {64 * 4, rows * 64 * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NL_OK : NL_ERR_CUDA;
}

inline int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Number of kernels this library has launched (all devices, all threads).
void count_launch();
// This device's error word (bounded-wait timeouts, guards), read by nl_get_device_error.
int* device_error_word();

inline int launch_status() {
  count_launch();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? NL_OK : NL_ERR_LAUNCH;
}

// Programmatic dependent launch for every kernel of this library (each one
// executes griddepcontrol.wait before its first global-memory access), so a
// kernel's launch and prologue overlap the tail of the one before it on the
// stream.  NL_PDL=0 turns it off.
inline bool pdl_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* e = getenv("NL_PDL");
    on = (e && e[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// Launch `kern` with the library's launch attributes (PDL, and a cluster
// dimension when cluster_x > 1).  A failed launch is also the runtime's last
// error, which the launch_status() that follows every launch reports.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                 int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_x > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster_x;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace nl
