// safetensors -> detwgt value conversion on the GPU (model ingestion).
//
// Restates f32_to_wgt (det_num/convert.rs:77-93: round half to even of
// x * 2^16, saturated to i32, non-finite values rejected) over a whole tensor,
// with the per-row mass sum |w| that gemma-det-num-wgt-converter's overflow
// bound checks (tools/gemma-det-num-wgt-converter/main.rs:346-388) and the
// "every value fits i16" test of its width selection.  Byte work bound by
// HBM: one block per row, values decoded from F32, BF16 or F16.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "kernels.h"

namespace rdet {

namespace {

__device__ __forceinline__ float decode_value(const void* src, uint64_t i, int dtype) {
  if (dtype == kSrcF32) return __uint_as_float(static_cast<const uint32_t*>(src)[i]);
  const uint16_t h = static_cast<const uint16_t*>(src)[i];
  if (dtype == kSrcBF16) return __uint_as_float((uint32_t)h << 16);
  return __half2float(__ushort_as_half(h));
}

// f32_to_wgt: x * 2^16 is exact in float32 (an exponent shift; beyond the
// float32 range it is an infinity of the right sign, which saturates), rintf
// rounds half to even, and every float32 of magnitude below 2^31 is an
// integer the conversion keeps.
__device__ __forceinline__ int32_t f32_to_wgt(float x) {
  const float y = rintf(x * 65536.0f);
  if (y >= 2147483648.0f) return INT32_MAX;
  if (y <= -2147483648.0f) return INT32_MIN;
  return (int32_t)y;
}

__global__ void __launch_bounds__(256) convert_wgt_kernel(const void* src, int dtype, uint64_t rows,
                                                          uint64_t row_len, int32_t* out, uint64_t* row_mass,
                                                          uint32_t* stats) {
  __shared__ uint64_t part[8];
  uint32_t nonfinite = 0, wide = 0;
  for (uint64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    uint64_t mass = 0;
    const uint64_t base = r * row_len;
    for (uint64_t k = threadIdx.x; k < row_len; k += blockDim.x) {
      const float x = decode_value(src, base + k, dtype);
      int32_t b = 0;
      if (isfinite(x)) b = f32_to_wgt(x);
      else ++nonfinite;
      out[base + k] = b;
      // |INT32_MIN| is 2^31 as an unsigned magnitude
      mass += b < 0 ? (uint64_t)(0u - (uint32_t)b) : (uint64_t)b;
      wide |= (b < -32768 || b > 32767) ? 1u : 0u;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mass += __shfl_xor_sync(0xffffffffu, mass, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = mass;
    __syncthreads();
    if (threadIdx.x == 0) {
      uint64_t t = 0;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
      row_mass[r] = t;
    }
    __syncthreads();
  }
  if (nonfinite) atomicAdd(&stats[0], nonfinite);
  if (wide) atomicOr(&stats[1], 1u);
}

}  // namespace

void launch_convert_wgt(const void* src, int dtype, uint64_t rows, uint64_t row_len, int32_t* out,
                        uint64_t* row_mass, uint32_t* stats, cudaStream_t s) {
  const uint64_t grid = rows < (uint64_t)sm_count() * 16 ? rows : (uint64_t)sm_count() * 16;
  if (grid == 0) return;
  convert_wgt_kernel<<<(unsigned)grid, 256, 0, s>>>(src, dtype, rows, row_len, out, row_mass, stats);
}

}  // namespace rdet
