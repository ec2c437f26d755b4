// knn_prep.cu -- row conversion + norms, used at build time for the dataset
// and per search for the queries.
//
// Replaces the reference's host loops that cast the dataset and queries to
// fp16 (src/metal_context.mm:164-166,195-196) and compute fp32 row norms
// (compute_row_norms, src/metal_context.mm:127-137).  Two deliberate
// differences: the work runs on the GPU (one warp per row, coalesced,
// 16-byte vector loads/stores when the row layout allows), and the norm is
// taken over the fp16-ROUNDED values, so |q|^2 + |x|^2 - 2 q.x is the exact
// expansion of the squared distance between the stored vectors.
//
// Output rows have leading dimension ld >= dim (a multiple of 8 halves, so
// every row starts on a 16-byte boundary as TMA requires); the pad columns
// are written as zeros and contribute nothing to dot products or norms.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "knn_internal.h"

namespace knn {

namespace {

template <bool kHalfIn>
__device__ __forceinline__ float load_elem(const void* in, int64_t i) {
  if constexpr (kHalfIn) {
    return __half2float(static_cast<const __half*>(in)[i]);
  } else {
    return static_cast<const float*>(in)[i];
  }
}

// One warp per row, grid-stride over rows.  `vec` selects the 8-wide path:
// dim % 8 == 0 and the input base 16-byte aligned.
template <bool kHalfIn>
__global__ void convert_rows_kernel(const void* __restrict__ in, int64_t rows, int64_t rows_out,
                                    int64_t dim, __half* __restrict__ out, int64_t ld,
                                    float* __restrict__ norms, bool vec,
                                    uint32_t* __restrict__ fill, int64_t fill_n,
                                    uint32_t* __restrict__ epoch, bool spread) {
  // Let the next kernel (the scan) be scheduled now: its dataset loads do
  // not depend on this kernel, and it waits before reading the queries.
  // This kernel is itself a programmatic dependent of the previous search's
  // kernels, which may still read `out`: wait for them before writing.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // per-search state: the exchange epoch (read by the merge kernels of this
  // search after their own griddepcontrol.wait) and the scan's shared
  // per-query bounds
  if (epoch && blockIdx.x == 0 && threadIdx.x == 0) *epoch += 1u;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < fill_n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    fill[i] = 0xFFFFFFFFu;
  const int lane = threadIdx.x & 31;
  const int64_t warps_per_block = blockDim.x >> 5;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * warps_per_block + (threadIdx.x >> 5);
  const int64_t step = static_cast<int64_t>(gridDim.x) * warps_per_block;
  for (int64_t r = first; r < rows_out; r += step) {
    float acc = 0.0f;
    __half* orow = out + r * ld;
    // the input row this output row holds (spread: see spread_query_row)
    int64_t src = r;
    if (spread) {
      const int64_t lr = r % kQueryRows, l = lr % 32;
      src = l < 8 ? r / kQueryRows * 32 + 4 * l + lr / 32 : rows;
    }
    if (src >= rows) {
      // padding row: zeros (keeps whole TMA boxes inside the allocation)
      for (int64_t c = lane; c < ld; c += 32) orow[c] = __float2half_rn(0.0f);
    } else if (vec) {
      const int64_t groups = dim / 8;
      for (int64_t g = lane; g < groups; g += 32) {
        float v[8];
        if constexpr (kHalfIn) {
          const uint4 raw = reinterpret_cast<const uint4*>(static_cast<const __half*>(in) +
                                                           src * dim)[g];
          const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(h[j]);
            v[2 * j] = f.x;
            v[2 * j + 1] = f.y;
          }
        } else {
          const float4* f4 = reinterpret_cast<const float4*>(static_cast<const float*>(in) +
                                                             src * dim) + 2 * g;
          const float4 a = f4[0];
          const float4 b = f4[1];
          v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
          v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        }
        uint4 packed;
        __half2* h2 = reinterpret_cast<__half2*>(&packed);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __half2 h = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
          h2[j] = h;
          const float2 f = __half22float2(h);
          acc = fmaf(f.x, f.x, acc);
          acc = fmaf(f.y, f.y, acc);
        }
        reinterpret_cast<uint4*>(orow)[g] = packed;
      }
      // zero padding [dim, ld): dim is a multiple of 8 here
      for (int64_t c = dim + lane; c < ld; c += 32) orow[c] = __float2half_rn(0.0f);
    } else {
      for (int64_t c = lane; c < ld; c += 32) {
        __half h = __float2half_rn(0.0f);
        if (c < dim) {
          h = __float2half_rn(load_elem<kHalfIn>(in, src * dim + c));
          const float f = __half2float(h);
          acc = fmaf(f, f, acc);
        }
        orow[c] = h;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0 && src < rows) norms[src] = acc;
  }
}

}  // namespace

cudaError_t launch_convert_rows(const void* in, bool in_is_half, int64_t rows, int64_t rows_out,
                                int64_t dim, __half* out, int64_t ld, float* norms,
                                cudaStream_t stream, uint32_t* fill, int64_t fill_n,
                                uint32_t* epoch, bool spread) {
  if (rows_out < rows) rows_out = rows;
  if (rows_out <= 0) return cudaSuccess;
  const bool vec = (dim % 8 == 0) && ((reinterpret_cast<uintptr_t>(in) & 15u) == 0) &&
                   ((reinterpret_cast<uintptr_t>(out) & 15u) == 0) && (ld % 8 == 0);
  constexpr int kThreads = 256;
  const int64_t warps_needed = rows_out;
  int64_t blocks = (warps_needed + (kThreads / 32) - 1) / (kThreads / 32);
  if (blocks > 148 * 16) blocks = 148 * 16;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(kThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (in_is_half)
    return cudaLaunchKernelEx(&cfg, convert_rows_kernel<true>, in, rows, rows_out, dim, out, ld,
                              norms, vec, fill, fill ? fill_n : int64_t(0), epoch, spread);
  return cudaLaunchKernelEx(&cfg, convert_rows_kernel<false>, in, rows, rows_out, dim, out, ld,
                            norms, vec, fill, fill ? fill_n : int64_t(0), epoch, spread);
}

}  // namespace knn
