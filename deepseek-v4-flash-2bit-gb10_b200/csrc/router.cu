// Router for the routed experts: topk_w, topk_ids = top-k(softmax(x . W_r)) per token, the
// selected probabilities as weights (not renormalised). This is the routing the benchmark
// configurations specify; in vLLM it is the router step that runs just before the MoE method (the
// reference plugin receives its output). Two kernels chained by programmatic dependent launch:
//
//   logits   G CTAs, CTA b owns hidden rows [b*H/G, (b+1)*H/G): for every token and expert it
//            writes the fp32 partial dot product over its rows (W_r rows are read coalesced;
//            x is staged in shared memory) into part[b][n][e].
//   select   one CTA per token: sums the partials in slice order (deterministic), softmax over the
//            experts; every warp takes the top k of its experts with k shuffle argmax rounds (value
//            descending, index ascending on ties), and warp 0 merges the warps' candidates the same
//            way.
#include "vq2_common.cuh"

namespace vq2 {

constexpr int RT_THREADS = 256;
constexpr int RT_MAX_E = 1024;
constexpr int RT_MAX_N = 64;
constexpr int RT_ROWS = 64;            // hidden rows per logits CTA
constexpr int RT_MAX_K = 64;

__global__ void __launch_bounds__(RT_THREADS) router_logits_kernel(const void* __restrict__ x, int x_dtype,
                                                                   const __nv_bfloat16* __restrict__ wr, int N, int H,
                                                                   int E, float* __restrict__ part) {
  pdl_launch_dependents();             // the select kernel waits for this grid before reading part
  __shared__ float xs[RT_MAX_N][RT_ROWS];
  const int b = blockIdx.x, h0 = b * RT_ROWS;
  for (int i = threadIdx.x; i < N * RT_ROWS; i += RT_THREADS) {
    const int n = i / RT_ROWS, r = i % RT_ROWS;
    xs[n][r] = load_act(x, x_dtype, (size_t)n * H + h0 + r);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += RT_THREADS) {
    float w[RT_ROWS];
#pragma unroll
    for (int r = 0; r < RT_ROWS; ++r) w[r] = __bfloat162float(wr[(size_t)(h0 + r) * E + e]);
    for (int n = 0; n < N; ++n) {
      float acc = 0.f;
#pragma unroll
      for (int r = 0; r < RT_ROWS; ++r) acc = fmaf(xs[n][r], w[r], acc);
      part[((size_t)b * N + n) * E + e] = acc;
    }
  }
}

// CTA-wide argmax of (v, i): larger value first, smaller index on ties.
__device__ __forceinline__ void rt_better(float& v, int& i, float v2, int i2) {
  if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

__global__ void __launch_bounds__(RT_THREADS) router_select_kernel(const float* __restrict__ part, int G, int E, int k,
                                                                   int N, int32_t* __restrict__ ids,
                                                                   float* __restrict__ wts) {
  pdl_wait();
  __shared__ float p[RT_MAX_E];
  __shared__ float red_v[RT_THREADS / 32];
  const int n = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float m = -INFINITY;
  for (int e = threadIdx.x; e < E; e += RT_THREADS) {
    float l = 0.f;
    for (int b = 0; b < G; ++b) l += part[((size_t)b * N + n) * E + e];
    p[e] = l;
    m = fmaxf(m, l);
  }
  m = warp_max(m);
  if (lane == 0) red_v[warp] = m;
  __syncthreads();
  m = red_v[0];
  for (int w = 1; w < RT_THREADS / 32; ++w) m = fmaxf(m, red_v[w]);
  __syncthreads();
  float s = 0.f;
  for (int e = threadIdx.x; e < E; e += RT_THREADS) {
    const float q = expf(p[e] - m);
    p[e] = q;
    s += q;
  }
  s = warp_sum(s);
  if (lane == 0) red_v[warp] = s;
  __syncthreads();
  s = 0.f;
  for (int w = 0; w < RT_THREADS / 32; ++w) s += red_v[w];
  __syncthreads();
  const float inv = 1.f / s;
  for (int e = threadIdx.x; e < E; e += RT_THREADS) p[e] *= inv;
  __syncthreads();
  // stage 1: each warp's top k over the experts e = warp*32 + lane + 256*i (k shuffle rounds)
  __shared__ float cand_v[RT_THREADS / 32][RT_MAX_K];
  __shared__ int cand_i[RT_THREADS / 32][RT_MAX_K];
  for (int j = 0; j < k; ++j) {
    float v = -1.f;
    int i = 0x7FFFFFFF;
    for (int e = threadIdx.x; e < E; e += RT_THREADS) rt_better(v, i, p[e], e);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) rt_better(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
    if (lane == 0) { cand_v[warp][j] = v; cand_i[warp][j] = i; }
    if (i != 0x7FFFFFFF && (i % RT_THREADS) == threadIdx.x) p[i] = -2.f;   // owner drops it
    __syncwarp();
  }
  __syncthreads();
  // stage 2: warp 0 merges the warps' candidates (k per warp) the same way
  if (warp == 0) {
    constexpr int NC = (RT_THREADS / 32) * RT_MAX_K / 32;   // candidates per lane (at most)
    float cv[NC];
    int ci[NC];
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      const int c = lane + 32 * q, w = c / RT_MAX_K, j = c % RT_MAX_K;
      const bool ok = j < k;
      cv[q] = ok ? cand_v[w][j] : -1.f;
      ci[q] = ok ? cand_i[w][j] : 0x7FFFFFFF;
    }
    for (int j = 0; j < k; ++j) {
      float v = -1.f;
      int i = 0x7FFFFFFF;
#pragma unroll
      for (int q = 0; q < NC; ++q) rt_better(v, i, cv[q], ci[q]);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) rt_better(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
      if (lane == 0) { ids[(size_t)n * k + j] = i; wts[(size_t)n * k + j] = v; }
#pragma unroll
      for (int q = 0; q < NC; ++q)
        if (ci[q] == i) cv[q] = -2.f;     // every id appears once among the candidates
    }
  }
}

}  // namespace vq2

using namespace vq2;

extern "C" size_t vq2_router_workspace_size(int N, int H, int E) {
  if (N <= 0 || H <= 0 || E <= 0) return 0;
  return (size_t)(H / RT_ROWS) * N * E * sizeof(float) + 256;
}

extern "C" int vq2_router_topk(const void* x, int x_dtype, const void* w_r, int N, int H, int E, int k,
                               int32_t* topk_ids, float* topk_w, void* ws, size_t ws_bytes, void* stream) {
  if (!x || !w_r || !topk_ids || !topk_w) return VQ2_ERR_NULL;
  if (N <= 0 || N > RT_MAX_N || H <= 0 || H % RT_ROWS || E <= 0 || E > RT_MAX_E || k <= 0 || k > E || k > RT_MAX_K)
    return VQ2_ERR_SHAPE;
  if (x_dtype < 0 || x_dtype > 2) return VQ2_ERR_DTYPE;
  if (!ws || ws_bytes < vq2_router_workspace_size(N, H, E)) return VQ2_ERR_WORKSPACE;
  float* part = (float*)(((uintptr_t)ws + 255) & ~(uintptr_t)255);
  const int G = H / RT_ROWS;
  cudaStream_t st = (cudaStream_t)stream;
  router_logits_kernel<<<G, RT_THREADS, 0, st>>>(x, x_dtype, (const __nv_bfloat16*)w_r, N, H, E, part);
  if (cudaGetLastError() != cudaSuccess) return VQ2_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(N);
  cfg.blockDim = dim3(RT_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, router_select_kernel, (const float*)part, G, E, k, N, topk_ids, topk_w) != cudaSuccess)
    return VQ2_ERR_CUDA;
  return VQ2_OK;
}
