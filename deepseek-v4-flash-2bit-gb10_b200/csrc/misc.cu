// Small elementwise kernels of the path and the library's status / error entry points:
//   per-row fp8 e4m3 quantisation (reference vq2_vllm/kernels/ds4_vq2_cuda.py:8-32),
//   group-64 Hadamard of rows       (reference vq2_vllm/kernels/vq2_kernel.py:188-195).
#include <cuda_fp8.h>
#include "vq2_common.cuh"

namespace vq2 {

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = l < nw ? red[l] : 0.f;
    v = warp_max(v);
    if (l == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

// one CTA per row: s = 448 / max(amax, 1e-6); q = e4m3(x * s) (round-to-nearest-even, saturating);
// inv = 1 / s — the reference's _quant_fp8_rows (ds4_vq2_cuda.py:11-23).
__global__ void quant_fp8_rows_kernel(const float* __restrict__ x, int cols, uint8_t* __restrict__ q,
                                      float* __restrict__ inv) {
  __shared__ float red[33];
  const float* xr = x + (size_t)blockIdx.x * cols;
  float amax = 0.f;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) amax = fmaxf(amax, fabsf(xr[c]));
  amax = block_max(amax, red);
  const float s = 448.0f / fmaxf(amax, 1e-6f);
  if (threadIdx.x == 0) inv[blockIdx.x] = 1.0f / s;
  uint8_t* qr = q + (size_t)blockIdx.x * cols;
  for (int c = threadIdx.x; c < cols; c += blockDim.x)
    qr[c] = (uint8_t)__nv_cvt_float_to_fp8(xr[c] * s, __NV_SATFINITE, __NV_E4M3);
}

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f(float v) { return v; }
template <> __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f(float v) { return v; }
template <> __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }

// one warp per 64-group: element lane + 32 r; shuffle butterflies for strides < 32.
template <typename TI, typename TO>
__global__ void hadamard_rows_kernel(const TI* __restrict__ x, TO* __restrict__ y, long ngroups) {
  const long g = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (g >= ngroups) return;
  const int lane = threadIdx.x & 31;
  float a = to_f(x[g * 64 + lane]), b = to_f(x[g * 64 + 32 + lane]);
  float t = a + b;
  b = a - b;
  a = t;
#pragma unroll
  for (int len = 16; len >= 1; len >>= 1) {
    const float pa = __shfl_xor_sync(0xffffffffu, a, len), pb = __shfl_xor_sync(0xffffffffu, b, len);
    a = (lane & len) ? (pa - a) : (a + pa);
    b = (lane & len) ? (pb - b) : (b + pb);
  }
  y[g * 64 + lane] = from_f<TO>(a * 0.125f);
  y[g * 64 + 32 + lane] = from_f<TO>(b * 0.125f);
}

template <typename TI>
static void launch_had(const void* x, void* y, int odt, long ng, cudaStream_t st) {
  const int wpb = 8;
  const long blocks = (ng + wpb - 1) / wpb;
  if (odt == VQ2_DT_BF16)
    hadamard_rows_kernel<TI, __nv_bfloat16><<<blocks, wpb * 32, 0, st>>>((const TI*)x, (__nv_bfloat16*)y, ng);
  else if (odt == VQ2_DT_F16)
    hadamard_rows_kernel<TI, __half><<<blocks, wpb * 32, 0, st>>>((const TI*)x, (__half*)y, ng);
  else
    hadamard_rows_kernel<TI, float><<<blocks, wpb * 32, 0, st>>>((const TI*)x, (float*)y, ng);
}

}  // namespace vq2

using namespace vq2;

extern "C" int vq2_quant_fp8_rows(const float* x, int rows, int cols, uint8_t* out, float* inv, void* stream) {
  if (!x || !out || !inv) return VQ2_ERR_NULL;
  if (rows < 0 || cols <= 0) return VQ2_ERR_SHAPE;
  if (rows == 0) return VQ2_OK;
  quant_fp8_rows_kernel<<<rows, 256, 0, (cudaStream_t)stream>>>(x, cols, out, inv);
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}

extern "C" int vq2_hadamard_rows(const void* x, int idt, void* y, int odt, long rows, int cols, void* stream) {
  if (!x || !y) return VQ2_ERR_NULL;
  if (rows < 0 || cols <= 0 || cols % 64) return VQ2_ERR_SHAPE;
  if (idt < 0 || idt > 2 || odt < 0 || odt > 2) return VQ2_ERR_DTYPE;
  if (rows == 0) return VQ2_OK;
  const long ng = rows * (cols / 64);
  cudaStream_t st = (cudaStream_t)stream;
  if (idt == VQ2_DT_BF16) launch_had<__nv_bfloat16>(x, y, odt, ng, st);
  else if (idt == VQ2_DT_F16) launch_had<__half>(x, y, odt, ng, st);
  else launch_had<float>(x, y, odt, ng, st);
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}

extern "C" int vq2_device_status(int reset) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return VQ2_ERR_CUDA;
  if (cudaMemcpyFromSymbol(&v, g_status, sizeof(int)) != cudaSuccess) return VQ2_ERR_CUDA;
  if (reset) {
    int z = 0;
    if (cudaMemcpyToSymbol(g_status, &z, sizeof(int)) != cudaSuccess) return VQ2_ERR_CUDA;
  }
  return v;
}

extern "C" const char* vq2_strerror(int code) {
  switch (code) {
    case VQ2_OK: return "ok";
    case VQ2_ERR_NULL: return "vq2: a required pointer is NULL";
    case VQ2_ERR_SHAPE: return "vq2: unsupported or inconsistent dimensions";
    case VQ2_ERR_ALIGN: return "vq2: pointer not 16-byte aligned";
    case VQ2_ERR_DTYPE: return "vq2: unknown dtype code";
    case VQ2_ERR_WORKSPACE: return "vq2: workspace missing or too small";
    case VQ2_ERR_TOO_MANY_PAIRS: return "vq2: decode path supports at most VQ2_DECODE_MAX_PAIRS token-expert pairs";
    case VQ2_ERR_CUDA: return "vq2: CUDA runtime call failed";
    case VQ2_ERR_TIMEOUT: return "vq2: a bounded device wait timed out";
    case VQ2_ERR_NO_DEVICE: return "vq2: no CUDA device";
    case VQ2_ERR_NOALLOC_LIMIT: return "vq2: vq2_decode_noalloc needs more scratch than VQ2_NOALLOC_SCRATCH_BYTES (2 MiB); use vq2_decode with a workspace";
    default: return "vq2: unknown error";
  }
}

extern "C" int vq2_version(void) { return 1; }
