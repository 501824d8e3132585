// K6 — shared expert of the decode step: a dense bf16 SiLU-gated MLP beside the routed experts
//   out[n] (+)= W2 . (silu(Wg . x[n]) * (Wu . x[n]))
// with w13 = [Wg; Wu] bf16 [2*Is][H] and w2 bf16 [H][Is]. In the model this plugin serves, vLLM
// runs the shared expert beside the MoE method (the method's `apply` receives and ignores it,
// reference vq2_vllm/__init__.py:197-198); this is the same layer as two HBM-streaming GEMV
// kernels chained by programmatic dependent launch, so a decode step can add it onto the routed
// output on the same stream without a host round trip:
//   gateup  issues the first weight chunks of its rows, waits for its predecessor (x and `out`
//           may come from it), releases the dependent launch, stages x; every warp takes (gate
//           row r, up row r) pairs: 16-byte non-caching loads of both rows, 8 chunks (8 KB) in
//           flight per warp, fp32 dot products against x staged in shared memory as fp32, warp
//           reduction, inter[n][r] = silu(g) * u in fp32.
//   down    starts while gateup runs: each warp loads the first chunks of its two W2 rows into
//           registers BEFORE waiting for gateup, then stages inter in shared memory and finishes
//           its rows; out[n][h] = (accumulate ? out[n][h] : 0) + sum.
// Both kernels stream their weights once: 2*Is*H*2 + H*Is*2 bytes per call (50.3 MB at H=4096,
// Is=2048), which is the HBM roofline of the layer.
#include "vq2_common.cuh"

namespace vq2 {

constexpr int SE_THREADS = 256;
constexpr int SE_WARPS = SE_THREADS / 32;
constexpr int SE_MAX_N = 8;
constexpr int SE_BATCH = 8;            // 16-byte chunks per row in flight per lane
constexpr int SE_CTAS_PER_SM = 2;

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// acc += <8 bf16 weights in w, 8 fp32 values at xs>
__device__ __forceinline__ float dot8_bf16(uint4 w, const float* xs, float acc) {
  const float4 a = *reinterpret_cast<const float4*>(xs);
  const float4 b = *reinterpret_cast<const float4*>(xs + 4);
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
  const float xv[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc = fmaf(__uint_as_float(u[i] << 16), xv[2 * i], acc);
    acc = fmaf(__uint_as_float(u[i] & 0xFFFF0000u), xv[2 * i + 1], acc);
  }
  return acc;
}

// dst[0 .. n) = fp32 of src (VQ2_DT_*), 16-byte loads; n a multiple of 8, src 16-byte aligned
__device__ __forceinline__ void stage_f32(float* dst, const void* src, int dt, int n) {
  if (dt == VQ2_DT_F32) {
    for (int i = threadIdx.x * 4; i < n; i += SE_THREADS * 4)
      *reinterpret_cast<float4*>(dst + i) = *reinterpret_cast<const float4*>(static_cast<const float*>(src) + i);
    return;
  }
  for (int i = threadIdx.x * 8; i < n; i += SE_THREADS * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(src) + i);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    float f[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (dt == VQ2_DT_BF16) {
        f[2 * j] = __uint_as_float(u[j] << 16);
        f[2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
      } else {
        const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&u[j]));
        f[2 * j] = h.x;
        f[2 * j + 1] = h.y;
      }
    }
    *reinterpret_cast<float4*>(dst + i) = make_float4(f[0], f[1], f[2], f[3]);
    *reinterpret_cast<float4*>(dst + i + 4) = make_float4(f[4], f[5], f[6], f[7]);
  }
}

__global__ void __launch_bounds__(SE_THREADS, SE_CTAS_PER_SM) shared_gateup_kernel(
    const void* __restrict__ x, int x_dtype, const __nv_bfloat16* __restrict__ w13, int N, int H, int Is,
    float* __restrict__ inter) {
  extern __shared__ __align__(16) float xs[];          // [N][H]
  const int lane = threadIdx.x & 31;
  const int nch = H / 256;                             // 16-byte chunks per lane per row
  const long long nw = (long long)gridDim.x * SE_WARPS;
  long long r = (long long)blockIdx.x * SE_WARPS + (threadIdx.x >> 5);
  uint4 wg[SE_BATCH], wu[SE_BATCH];
  // the weights depend on nothing earlier in the stream: fetch the first chunks of this warp's
  // first row pair before waiting for the predecessor and staging x
  if (r < Is) {
    const char* rg = reinterpret_cast<const char*>(w13 + (size_t)r * H) + lane * 16;
    const char* ru = reinterpret_cast<const char*>(w13 + (size_t)(r + Is) * H) + lane * 16;
#pragma unroll
    for (int c = 0; c < SE_BATCH; ++c) {
      if (c < nch) {
        wg[c] = ld_stream16(rg + (size_t)c * 512);
        wu[c] = ld_stream16(ru + (size_t)c * 512);
      }
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  stage_f32(xs, x, x_dtype, N * H);
  __syncthreads();
  bool first = true;
  for (; r < Is; r += nw) {
    const char* rg = reinterpret_cast<const char*>(w13 + (size_t)r * H) + lane * 16;
    const char* ru = reinterpret_cast<const char*>(w13 + (size_t)(r + Is) * H) + lane * 16;
    float g[SE_MAX_N], u[SE_MAX_N];
#pragma unroll
    for (int n = 0; n < SE_MAX_N; ++n) g[n] = u[n] = 0.f;
    for (int c0 = 0; c0 < nch; c0 += SE_BATCH) {
      if (!(first && c0 == 0)) {
#pragma unroll
        for (int c = 0; c < SE_BATCH; ++c) {
          if (c0 + c < nch) {
            wg[c] = ld_stream16(rg + (size_t)(c0 + c) * 512);
            wu[c] = ld_stream16(ru + (size_t)(c0 + c) * 512);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < SE_BATCH; ++c) {
        if (c0 + c < nch) {
          const int col = (c0 + c) * 256 + lane * 8;
#pragma unroll
          for (int n = 0; n < SE_MAX_N; ++n) {
            if (n < N) {
              g[n] = dot8_bf16(wg[c], xs + n * H + col, g[n]);
              u[n] = dot8_bf16(wu[c], xs + n * H + col, u[n]);
            }
          }
        }
      }
    }
    first = false;
#pragma unroll
    for (int n = 0; n < SE_MAX_N; ++n) {
      if (n < N) {
        const float gs = warp_sum(g[n]), us = warp_sum(u[n]);
        if (lane == 0) inter[(size_t)n * Is + r] = gs / (1.f + __expf(-gs)) * us;
      }
    }
  }
}

__global__ void __launch_bounds__(SE_THREADS, SE_CTAS_PER_SM) shared_down_kernel(
    const float* __restrict__ inter, const __nv_bfloat16* __restrict__ w2, int N, int H, int Is,
    float* __restrict__ out, int accumulate) {
  extern __shared__ __align__(16) float is_[];         // [N][Is]
  const int lane = threadIdx.x & 31;
  const int nch = Is / 256;
  const long long nunits = H / 2;                      // two W2 rows per warp unit
  const long long nw = (long long)gridDim.x * SE_WARPS;
  long long unit = (long long)blockIdx.x * SE_WARPS + (threadIdx.x >> 5);
  uint4 wa[SE_BATCH], wb[SE_BATCH];
  // prefetch the first chunks of this warp's first rows while the gate/up kernel still runs
  if (unit < nunits) {
    const char* ra = reinterpret_cast<const char*>(w2 + (size_t)(2 * unit) * Is) + lane * 16;
#pragma unroll
    for (int c = 0; c < SE_BATCH; ++c) {
      if (c < nch) {
        wa[c] = ld_stream16(ra + (size_t)c * 512);
        wb[c] = ld_stream16(ra + (size_t)Is * 2 + (size_t)c * 512);
      }
    }
  }
  pdl_wait();
  stage_f32(is_, inter, VQ2_DT_F32, N * Is);
  __syncthreads();
  bool first = true;
  for (; unit < nunits; unit += nw) {
    const char* ra = reinterpret_cast<const char*>(w2 + (size_t)(2 * unit) * Is) + lane * 16;
    float a[SE_MAX_N], b[SE_MAX_N];
#pragma unroll
    for (int n = 0; n < SE_MAX_N; ++n) a[n] = b[n] = 0.f;
    for (int c0 = 0; c0 < nch; c0 += SE_BATCH) {
      if (!(first && c0 == 0)) {
#pragma unroll
        for (int c = 0; c < SE_BATCH; ++c) {
          if (c0 + c < nch) {
            wa[c] = ld_stream16(ra + (size_t)(c0 + c) * 512);
            wb[c] = ld_stream16(ra + (size_t)Is * 2 + (size_t)(c0 + c) * 512);
          }
        }
      }
#pragma unroll
      for (int c = 0; c < SE_BATCH; ++c) {
        if (c0 + c < nch) {
          const int col = (c0 + c) * 256 + lane * 8;
#pragma unroll
          for (int n = 0; n < SE_MAX_N; ++n) {
            if (n < N) {
              a[n] = dot8_bf16(wa[c], is_ + n * Is + col, a[n]);
              b[n] = dot8_bf16(wb[c], is_ + n * Is + col, b[n]);
            }
          }
        }
      }
    }
    first = false;
#pragma unroll
    for (int n = 0; n < SE_MAX_N; ++n) {
      if (n < N) {
        const float as = warp_sum(a[n]), bs = warp_sum(b[n]);
        if (lane == 0) {
          float* o = out + (size_t)n * H + 2 * unit;
          if (accumulate == 2) {          // concurrent with other writers of `out`: fp32 atomics
            atomicAdd(o, as);
            atomicAdd(o + 1, bs);
          } else {
            o[0] = accumulate ? o[0] + as : as;
            o[1] = accumulate ? o[1] + bs : bs;
          }
        }
      }
    }
  }
}

constexpr int SE_SMEM_CAP = 200 * 1024;   // dynamic shared memory of either kernel (x or inter as fp32)

// grid of a kernel whose warps take `warps` row units: at most SE_CTAS_PER_SM CTAs per SM of the
// `sms` SMs it may use (all of them when sms <= 0)
inline int se_grid(long long warps, int sms = 0) {
  const long long b = (warps + SE_WARPS - 1) / SE_WARPS;
  const long long nsm = sms > 0 ? sms : std::max(device_sm_count(), 1);
  return (int)std::min<long long>(std::max<long long>(b, 1), nsm * SE_CTAS_PER_SM);
}

// Validation of a shared-expert call (0 if it can run).
inline int se_check(const void* x, int x_dtype, const void* w13, const void* w2, int N, int H, int Is,
                    const float* out) {
  if (!x || !w13 || !w2 || !out) return VQ2_ERR_NULL;
  if (N <= 0 || N > SE_MAX_N || H <= 0 || Is <= 0 || H % 256 || Is % 256 || H % 2) return VQ2_ERR_SHAPE;
  if ((size_t)N * H * sizeof(float) > (size_t)SE_SMEM_CAP || (size_t)N * Is * sizeof(float) > (size_t)SE_SMEM_CAP)
    return VQ2_ERR_SHAPE;
  if (x_dtype < 0 || x_dtype > 2) return VQ2_ERR_DTYPE;
  if ((uintptr_t)w13 % 16 || (uintptr_t)w2 % 16 || (uintptr_t)x % 16) return VQ2_ERR_ALIGN;
  return VQ2_OK;
}

// The two kernels on `stream` (inputs checked by se_check). accumulate: 0 write, 1 add, 2 add
// with fp32 atomics; sms > 0 caps the grids to that many SMs' worth of CTAs.
inline int se_launch(const void* x, int x_dtype, const void* w13, const void* w2, int N, int H, int Is,
                     float* out, int accumulate, float* inter, cudaStream_t stream, int sms) {
  // The dynamic shared-memory limit is raised once per device to the cap every call fits in, so
  // calls with different N (other threads, captured graphs) never lower it under one another.
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VQ2_ERR_NO_DEVICE;
  static bool attr_set[64];
  if (!attr_set[dev]) {
    if (cudaFuncSetAttribute(shared_gateup_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SE_SMEM_CAP) != cudaSuccess ||
        cudaFuncSetAttribute(shared_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SE_SMEM_CAP) != cudaSuccess)
      return VQ2_ERR_CUDA;
    attr_set[dev] = true;
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(SE_THREADS);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.gridDim = dim3(se_grid(Is, sms));
  cfg.dynamicSmemBytes = (size_t)N * H * sizeof(float);
  if (cudaLaunchKernelEx(&cfg, shared_gateup_kernel, x, x_dtype, (const __nv_bfloat16*)w13, N, H, Is, inter) !=
      cudaSuccess)
    return VQ2_ERR_CUDA;
  cfg.gridDim = dim3(se_grid(H / 2, sms));
  cfg.dynamicSmemBytes = (size_t)N * Is * sizeof(float);
  if (cudaLaunchKernelEx(&cfg, shared_down_kernel, (const float*)inter, (const __nv_bfloat16*)w2, N, H, Is, out,
                         accumulate) != cudaSuccess)
    return VQ2_ERR_CUDA;
  return VQ2_OK;
}

}  // namespace vq2

using namespace vq2;

extern "C" size_t vq2_shared_expert_workspace_size(int N, int Is) {
  if (N <= 0 || Is <= 0) return 0;
  return (size_t)N * Is * sizeof(float) + 256;
}

extern "C" int vq2_shared_expert(const void* x, int x_dtype, const void* w13, const void* w2, int N, int H, int Is,
                                 float* out, int accumulate, void* ws, size_t ws_bytes, void* stream) {
  const int rc = se_check(x, x_dtype, w13, w2, N, H, Is, out);
  if (rc) return rc;
  if (!ws || ws_bytes < vq2_shared_expert_workspace_size(N, Is)) return VQ2_ERR_WORKSPACE;
  float* inter = (float*)(((uintptr_t)ws + 255) & ~(uintptr_t)255);
  return se_launch(x, x_dtype, w13, w2, N, H, Is, out, accumulate ? 1 : 0, inter, (cudaStream_t)stream, 0);
}

// ------------------------------------------------------------------ routed + shared, co-scheduled
// The routed decode kernels are issue bound (codebook gathers) and leave HBM bandwidth unused; the
// shared expert is a pure weight stream. Running the shared expert's kernels on a partition of the
// SMs while the routed kernels hold the rest overlaps the two: the output is zeroed once, the
// routed grids run on (SMs - shared_sms) CTAs and add with their fp32 atomics, and the shared
// kernels run concurrently on a second stream (this library's, one per device, forked from and
// joined back into the caller's stream with events) on shared_sms SMs' worth of CTAs, adding with
// fp32 atomics. A host lock per device keeps concurrent callers' fork/join pairs apart.
#include <mutex>

namespace vq2 {
struct CoSched {
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  std::mutex mu;
};
static CoSched g_cosched[64];
}  // namespace vq2

extern "C" size_t vq2_decode_with_shared_workspace_size(int N, int topk, int H, int I, int Is) {
  const size_t a = (vq2_decode_workspace_size(N, topk, H, I) + 255) & ~(size_t)255;
  return a + vq2_shared_expert_workspace_size(N, Is);
}

extern "C" int vq2_decode_with_shared(const vq2_moe_args* a, const void* sw13, const void* sw2, int Is, int shared_sms,
                                      void* ws, size_t ws_bytes, void* stream) {
  if (!a) return VQ2_ERR_NULL;
  int rc = se_check(a->x, a->x_dtype, sw13, sw2, a->N, a->H, Is, a->out);
  if (rc) return rc;
  if (!ws || ws_bytes < vq2_decode_with_shared_workspace_size(a->N, a->topk, a->H, a->I, Is)) return VQ2_ERR_WORKSPACE;
  const size_t wa = (vq2_decode_workspace_size(a->N, a->topk, a->H, a->I) + 255) & ~(size_t)255;
  float* inter = (float*)((((uintptr_t)ws + wa) + 255) & ~(uintptr_t)255);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VQ2_ERR_NO_DEVICE;
  const int nsm = device_sm_count();
  if (nsm <= 0) return VQ2_ERR_CUDA;
  if (shared_sms <= 0) shared_sms = VQ2_SHARED_SMS_DEFAULT;
  if (shared_sms >= nsm) return VQ2_ERR_SHAPE;
  CoSched& cs = g_cosched[dev];
  std::lock_guard<std::mutex> lock(cs.mu);
  if (!cs.side) {
    if (cudaStreamCreateWithFlags(&cs.side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&cs.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&cs.join, cudaEventDisableTiming) != cudaSuccess)
      return VQ2_ERR_CUDA;
  }
  cudaStream_t s = (cudaStream_t)stream;
  if (cudaMemsetAsync(a->out, 0, (size_t)a->N * a->H * sizeof(float), s) != cudaSuccess) return VQ2_ERR_CUDA;
  if (cudaEventRecord(cs.fork, s) != cudaSuccess || cudaStreamWaitEvent(cs.side, cs.fork, 0) != cudaSuccess)
    return VQ2_ERR_CUDA;
  // routed first, so its one-CTA-per-SM grids take their SMs before the shared kernels' CTAs land
  DecEp ep = {};
  ep.keep_out = 1;
  rc = decode_launch(a, ws, wa, stream, ep, nsm - shared_sms);
  if (rc) return rc;
  rc = se_launch(a->x, a->x_dtype, sw13, sw2, a->N, a->H, Is, a->out, 2, inter, cs.side, shared_sms);
  if (rc) return rc;
  if (cudaEventRecord(cs.join, cs.side) != cudaSuccess || cudaStreamWaitEvent(s, cs.join, 0) != cudaSuccess)
    return VQ2_ERR_CUDA;
  return VQ2_OK;
}
