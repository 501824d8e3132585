// Expert-parallel token exchange over NVLink peer memory.
//
// The reference runs on one device; this is the exchange step of the B200 build's expert
// parallelism (experts partitioned over ranks, every rank applies its experts to every rank's
// decode tokens). Each rank owns one exchange region (layout in include/vq2_b200.h) that every
// other rank has mapped through a CUDA IPC handle, so the exchange is plain peer stores over
// NVLink plus one flag per (source, destination) pair:
//
//   dispatch               this rank's token rows, ids and weights -> slot `rank` of every rank's
//                          region, in VQ2_EP_CTAS slices (one CTA each, one flag each at every
//                          destination); CTA 0 waits (bounded) until every source's slices are here.
//   combine                the partial output rows of rank d's tokens -> slot `rank` of rank d's
//                          COMB (VQ2_EP_CTAS CTAs per destination, one flag each); every CTA waits
//                          for all sources, then sums its slice of the output over the slots in
//                          source order (deterministic).
//
// Steps are numbered by a counter in the region (EPOCH), advanced on the device by dispatch, so
// the calls carry no per-step host value and can be captured in a CUDA graph. Single buffering is
// safe: a rank writes a peer's slot for step s+1 only after that peer has finished step s (its
// combine of step s needs this rank's step-s partials, pushed after this rank's step-s decode,
// which consumed the step-s rows).
#include <cstring>
#include "vq2_common.cuh"

namespace vq2 {


// CTA-wide copy of `bytes` (a multiple of 16, both ends 16-byte aligned) to peer memory.
__device__ __forceinline__ void ep_copy16(uint8_t* dst, const uint8_t* src, size_t bytes) {
  const size_t n = bytes / 16;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) ((uint4*)dst)[i] = ((const uint4*)src)[i];
}
// The same for 4-byte multiples (ids / weights when k is not a multiple of 4).
__device__ __forceinline__ void ep_copy4(uint8_t* dst, const uint8_t* src, size_t bytes) {
  const size_t n = bytes / 4;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) ((uint32_t*)dst)[i] = ((const uint32_t*)src)[i];
}

// grid: C = ep_slices(N * row_x) CTAs. CTA c pushes slice c of this rank's rows, ids (narrowed to
// i32 when given as i64) and weights to every rank, then releases flag [rank][c] there. CTA 0 waits
// for all world x C flags here and then advances the step counter (it cannot finish before every
// CTA of this launch has released its flag to this rank, so every CTA reads the counter before it
// changes).
__global__ void __launch_bounds__(512) ep_dispatch_kernel(const uint8_t* __restrict__ x, const void* __restrict__ ids,
                                                          int ids_i64, const float* __restrict__ w, int N, int row_x,
                                                          int k, const uint64_t* __restrict__ peers, int world,
                                                          int rank, unsigned* my_dflag, unsigned* epoch) {
  // launched with programmatic dependent launch: the decode kernel behind may become resident now
  // (it waits for this grid); this grid waits for its predecessor (the previous step's combine,
  // which saw every rank's partials, so every peer has consumed the slots written here) first
  pdl_launch_dependents();
  pdl_wait();
  const int C = gridDim.x;
  const int c = blockIdx.x;
  const unsigned ep = *epoch + 1;
  const size_t xb = (size_t)N * row_x, ib = (size_t)N * k * 4;
  const bool v16 = (ib % 16) == 0;
  size_t xb0, xb1, ib0, ib1;
  ep_slice(xb, c, C, 16, xb0, xb1);
  ep_slice(ib, c, C, v16 ? 16 : 4, ib0, ib1);
  for (int p = 0; p < world; ++p) {
    const uint64_t* t = peers + p * EP_FIELDS;
    ep_copy16((uint8_t*)t[EP_X] + rank * xb + xb0, x + xb0, xb1 - xb0);
    if (ids_i64) {
      int32_t* dst = (int32_t*)((uint8_t*)t[EP_IDS] + rank * ib);
      for (size_t i = ib0 / 4 + threadIdx.x; i < ib1 / 4; i += blockDim.x) dst[i] = (int32_t)((const long long*)ids)[i];
    } else if (v16) {
      ep_copy16((uint8_t*)t[EP_IDS] + rank * ib + ib0, (const uint8_t*)ids + ib0, ib1 - ib0);
    } else {
      ep_copy4((uint8_t*)t[EP_IDS] + rank * ib + ib0, (const uint8_t*)ids + ib0, ib1 - ib0);
    }
    if (v16) ep_copy16((uint8_t*)t[EP_WT] + rank * ib + ib0, (const uint8_t*)w + ib0, ib1 - ib0);
    else ep_copy4((uint8_t*)t[EP_WT] + rank * ib + ib0, (const uint8_t*)w + ib0, ib1 - ib0);
  }
  __syncthreads();                       // every thread's stores precede the releases below
  if (threadIdx.x < world) {
    st_release_sys((unsigned*)peers[threadIdx.x * EP_FIELDS + EP_DFLAG] + rank * C + c, ep);
  }
  if (c == 0) {
    for (int f = threadIdx.x; f < world * C; f += blockDim.x) ep_wait_flag(my_dflag + f, ep);
    __syncthreads();
    if (threadIdx.x == 0) *epoch = ep;
  }
}

// grid: world x C CTAs, C = ep_slices(N * H * 4). CTA (d, c) pushes slice c of the partial rows of
// rank d's tokens into slot `rank` of rank d's COMB and releases flag [rank][c] there; then every
// CTA waits for all world x C flags here and sums its slice of the output over the source slots, in
// source order (deterministic).
__global__ void __launch_bounds__(512) ep_combine_kernel(const float* __restrict__ part, int N, int H,
                                                         const uint64_t* __restrict__ peers, int world, int rank,
                                                         const float* my_comb, unsigned* my_cflag,
                                                         const unsigned* epoch, float* __restrict__ out) {
  // launched with programmatic dependent launch behind the down kernel: resident early, it waits
  // for that grid (whose partials it pushes) before reading anything
  pdl_launch_dependents();
  pdl_wait();
  const int C = gridDim.x / world;
  const unsigned ep = *epoch;            // this step, advanced by the dispatch kernel
  const int d = blockIdx.x / C, c = blockIdx.x % C;
  const size_t nb = (size_t)N * H * 4;
  size_t b0, b1;
  ep_slice(nb, c, C, 16, b0, b1);
  ep_copy16((uint8_t*)peers[d * EP_FIELDS + EP_COMB] + rank * nb + b0,
            (const uint8_t*)(part + (size_t)d * N * H) + b0, b1 - b0);
  __syncthreads();
  if (threadIdx.x == 0) {
    st_release_sys((unsigned*)peers[d * EP_FIELDS + EP_CFLAG] + rank * C + c, ep);
  }
  for (int f = threadIdx.x; f < world * C; f += blockDim.x) ep_wait_flag(my_cflag + f, ep);
  __syncthreads();
  // this CTA's slice of the output; L2 loads (__ldcg) because the slots were written by other
  // GPUs since this SM last read them
  const size_t tot4 = (size_t)N * H / 4;
  const size_t per = (tot4 + gridDim.x - 1) / gridDim.x;
  const size_t b = (size_t)blockIdx.x * per, e = min(tot4, b + per);
  for (size_t i = b + threadIdx.x; i < e; i += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < world; ++s) {
      const float4 v = __ldcg((const float4*)my_comb + (size_t)s * tot4 + i);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    ((float4*)out)[i] = acc;
  }
}

}  // namespace vq2

using namespace vq2;

extern "C" int vq2_ep_alloc(size_t bytes, void** dev_ptr_out) {
  if (!dev_ptr_out || bytes == 0) return VQ2_ERR_NULL;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return VQ2_ERR_CUDA;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) { cudaFree(p); return VQ2_ERR_CUDA; }
  *dev_ptr_out = p;
  return VQ2_OK;
}

extern "C" int vq2_ep_free(void* dev_ptr) {
  return cudaFree(dev_ptr) == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}

extern "C" int vq2_ipc_get_handle(const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return VQ2_ERR_NULL;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return VQ2_ERR_CUDA;
  memcpy(handle_out, &h, sizeof(h));
  return VQ2_OK;
}

extern "C" int vq2_ipc_open(const void* handle, void** dev_ptr_out) {
  if (!handle || !dev_ptr_out) return VQ2_ERR_NULL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? VQ2_OK
                                                                                               : VQ2_ERR_CUDA;
}

extern "C" int vq2_ipc_close(void* dev_ptr) {
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}

extern "C" int vq2_ep_dispatch(const void* x, const void* ids, int ids_dtype, const float* w, int N, int row_x, int k,
                               const uint64_t* peers, int world, int rank, void* my_region, size_t off_dflag,
                               size_t off_epoch, void* stream) {
  if (!x || !ids || !w || !peers || !my_region) return VQ2_ERR_NULL;
  if (ids_dtype != VQ2_ID_I32 && ids_dtype != VQ2_ID_I64) return VQ2_ERR_DTYPE;
  if (N <= 0 || k <= 0 || row_x <= 0 || row_x % 16 || world < 1 || world > 64 || rank < 0 || rank >= world)
    return VQ2_ERR_SHAPE;
  if (((uintptr_t)x & 15) || ((uintptr_t)ids & 15) || ((uintptr_t)w & 15) || (off_dflag & 15) || (off_epoch & 15))
    return VQ2_ERR_ALIGN;
  uint8_t* r = (uint8_t*)my_region;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ep_slices((size_t)N * row_x));
  cfg.blockDim = dim3(512);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, ep_dispatch_kernel, (const uint8_t*)x, ids, (int)(ids_dtype == VQ2_ID_I64), w, N,
                            row_x, k, peers, world, rank, (unsigned*)(r + off_dflag), (unsigned*)(r + off_epoch)) ==
                 cudaSuccess
             ? VQ2_OK
             : VQ2_ERR_CUDA;
}

extern "C" int vq2_ep_combine(const float* part, int N, int H, const uint64_t* peers, int world, int rank,
                              void* my_region, size_t off_comb, size_t off_cflag, size_t off_epoch, float* out,
                              void* stream) {
  if (!part || !peers || !my_region || !out) return VQ2_ERR_NULL;
  if (N <= 0 || H <= 0 || H % 4 || world < 1 || world > 64 || rank < 0 || rank >= world) return VQ2_ERR_SHAPE;
  if (((uintptr_t)part & 15) || ((uintptr_t)out & 15) || (off_comb & 15) || (off_cflag & 15) || (off_epoch & 15))
    return VQ2_ERR_ALIGN;
  uint8_t* r = (uint8_t*)my_region;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(world * ep_slices((size_t)N * H * 4));
  cfg.blockDim = dim3(512);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, ep_combine_kernel, part, N, H, peers, world, rank, (const float*)(r + off_comb),
                            (unsigned*)(r + off_cflag), (const unsigned*)(r + off_epoch), out) == cudaSuccess
             ? VQ2_OK
             : VQ2_ERR_CUDA;
}
