// K3 — moe_align: stable sort of (token, slot) pairs by expert with per-expert padding to BM
// (replaces moe_align.moe_align / _moe_align_torch, reference vq2_vllm/kernels/moe_align.py:50-86;
// bit-exact with the torch version, whose rank within an expert is the pair order).
//
// Chunks of ALIGN_CHUNK pairs. count: per-chunk expert histogram (shared atomics); scan (one
// CTA): per-expert prefix over chunks, padded sizes, exclusive scan over experts, block -> expert
// table; place: each chunk ranks its pairs stably (warp match + per-warp counts, in order) and
// scatters. When M fits one chunk the three phases run in a single CTA (one launch).
#include "vq2_common.cuh"

namespace vq2 {

constexpr int ALIGN_THREADS = 1024;
constexpr int ALIGN_CHUNK = 8192;
constexpr int ALIGN_MAX_E = 1024;

__device__ __forceinline__ int clamp_e(int e, int E) { return e < 0 ? 0 : (e >= E ? E - 1 : e); }

// Local expert of a pair: id - base, clamped into [0, E) (reference semantics) or, with drop,
// -1 for ids outside [base, base + E) (expert parallelism: pairs owned by another device).
__device__ __forceinline__ int map_e(int id, int E, int base, int drop) {
  const int e = id - base;
  if (drop) return (e >= 0 && e < E) ? e : -1;
  return clamp_e(e, E);
}

// histogram of one chunk -> counts[chunk][E]
__device__ void align_count_chunk(const void* ids, int dt, long M, int E, int base, int drop, int chunk, int* counts,
                                  int* sh_cnt) {
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh_cnt[e] = 0;
  __syncthreads();
  const long b = (long)chunk * ALIGN_CHUNK, end = min(M, b + ALIGN_CHUNK);
  for (long m = b + threadIdx.x; m < end; m += blockDim.x) {
    const int e = map_e(load_id(ids, dt, m), E, base, drop);
    if (e >= 0) atomicAdd(&sh_cnt[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) counts[(long)chunk * E + e] = sh_cnt[e];
  __syncthreads();
}

// counts[c][e] -> absolute destination base of chunk c's first pair of expert e; block_e table.
__device__ void align_scan(int nchunks, int E, int BM, long Pmax, int* counts, int32_t* block_e, int* sh,
                           int2* ranges) {
  int* tot = sh;                     // [E] padded sizes, then offsets
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int c = 0; c < nchunks; ++c) {
      int v = counts[(long)c * E + e];
      counts[(long)c * E + e] = run;
      run += v;
    }
    tot[e] = ((run + BM - 1) / BM) * BM;
  }
  __syncthreads();
  if (threadIdx.x < 32) {            // exclusive scan of padded sizes by warp 0
    const int lane = threadIdx.x, per = (E + 31) / 32, b0 = lane * per;
    int local = 0;
    for (int e = b0; e < min(E, b0 + per); ++e) local += tot[e];
    int incl = local;
    for (int o = 1; o < 32; o <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    int run = incl - local;
    for (int e = b0; e < min(E, b0 + per); ++e) {
      int p = tot[e];
      tot[e] = run;
      run += p;
    }
    if (lane == 31) sh[ALIGN_MAX_E] = incl;   // used slots
  }
  __syncthreads();
  const long nblk = Pmax / BM;
  const int used_blocks = sh[ALIGN_MAX_E] / BM;
  // blocks inside an expert's region belong to it; trailing blocks map to E-1
  // (searchsorted(block_start, b, right=True) - 1, moe_align.py:82-84)
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int b0 = tot[e] / BM;
    const int b1 = (e + 1 < E) ? tot[e + 1] / BM : used_blocks;
    for (int b = b0; b < b1; ++b) block_e[b] = e;
    if (ranges) ranges[e] = make_int2(b0 * BM, (b1 - b0) * BM);   // expert e's padded slot range
  }
  for (long b = used_blocks + threadIdx.x; b < nblk; b += blockDim.x) block_e[b] = E - 1;
  for (int e = threadIdx.x; e < E; e += blockDim.x)
    for (int c = 0; c < nchunks; ++c) counts[(long)c * E + e] += tot[e];
  __syncthreads();
}

// stable placement of one chunk: rounds of blockDim pairs, in pair order
__device__ void align_place_chunk(const void* ids, int dt, long M, int k, int E, int ebase, int drop, int chunk,
                                  const int* base,
                                  int32_t* st, int32_t* ss, uint8_t* val, int* sh_run, int* sh_wc, int32_t* pslot) {
  const int nw = blockDim.x / 32, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh_run[e] = base[(long)chunk * E + e];
  __syncthreads();
  const long b = (long)chunk * ALIGN_CHUNK, end = min(M, b + ALIGN_CHUNK);
  for (long r0 = b; r0 < end; r0 += blockDim.x) {
    const long m = r0 + threadIdx.x;
    const int e0 = m < end ? map_e(load_id(ids, dt, m), E, ebase, drop) : -1;
    const bool act = e0 >= 0;
    const int e = act ? e0 : -1 - lane;   // inactive / dropped lanes: unique keys
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int lrank = __popc(peers & ((1u << lane) - 1));
    const bool leader = lrank == 0;
    if (act && leader) sh_wc[warp * E + e] = __popc(peers);
    __syncthreads();
    if (act) {
      int rank = sh_run[e] + lrank;
      for (int w = 0; w < warp; ++w) rank += sh_wc[w * E + e];
      st[rank] = (int32_t)(m / k);
      ss[rank] = (int32_t)(m % k);
      val[rank] = 1;
      if (pslot) pslot[m] = rank;
    } else if (pslot && m < end) {
      pslot[m] = -1;                      // pair owned by another device (dropped)
    }
    __syncthreads();
    if (act && leader) {
      atomicAdd(&sh_run[e], __popc(peers));
      sh_wc[warp * E + e] = 0;
    }
    __syncthreads();
  }
}

__device__ void zero_outputs(long Pmax, int32_t* st, int32_t* ss, uint8_t* val) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < Pmax; i += (long)gridDim.x * blockDim.x) {
    st[i] = 0;
    ss[i] = 0;
    val[i] = 0;
  }
}

struct AlignArgs {
  const void* ids; int dt; long M; int k; int E; int BM; int base; int drop; long Pmax; int nchunks;
  int32_t* st; int32_t* ss; uint8_t* val; int32_t* be; int* counts;
  int2* ranges;   // optional: per expert (first slot, padded slots)
  int32_t* pslot; // optional: per pair, its slot (-1 if dropped)
};

__global__ void __launch_bounds__(ALIGN_THREADS) align_single_kernel(AlignArgs a) {
  __shared__ int sh_a[ALIGN_MAX_E + 1];
  extern __shared__ int sh_wc[];          // [nwarps][E]
  zero_outputs(a.Pmax, a.st, a.ss, a.val);
  for (int i = threadIdx.x; i < (blockDim.x / 32) * a.E; i += blockDim.x) sh_wc[i] = 0;
  align_count_chunk(a.ids, a.dt, a.M, a.E, a.base, a.drop, 0, a.counts, sh_a);
  align_scan(1, a.E, a.BM, a.Pmax, a.counts, a.be, sh_a, a.ranges);
  align_place_chunk(a.ids, a.dt, a.M, a.k, a.E, a.base, a.drop, 0, a.counts, a.st, a.ss, a.val, sh_a, sh_wc, a.pslot);
}

__global__ void __launch_bounds__(ALIGN_THREADS) align_count_kernel(AlignArgs a) {
  __shared__ int sh_a[ALIGN_MAX_E];
  zero_outputs(a.Pmax, a.st, a.ss, a.val);
  align_count_chunk(a.ids, a.dt, a.M, a.E, a.base, a.drop, blockIdx.x, a.counts, sh_a);
}

__global__ void __launch_bounds__(ALIGN_THREADS) align_scan_kernel(AlignArgs a) {
  __shared__ int sh_a[ALIGN_MAX_E + 1];
  align_scan(a.nchunks, a.E, a.BM, a.Pmax, a.counts, a.be, sh_a, a.ranges);
}

__global__ void __launch_bounds__(ALIGN_THREADS) align_place_kernel(AlignArgs a) {
  __shared__ int sh_a[ALIGN_MAX_E];
  extern __shared__ int sh_wc[];
  for (int i = threadIdx.x; i < (blockDim.x / 32) * a.E; i += blockDim.x) sh_wc[i] = 0;
  __syncthreads();
  align_place_chunk(a.ids, a.dt, a.M, a.k, a.E, a.base, a.drop, blockIdx.x, a.counts, a.st, a.ss, a.val, sh_a, sh_wc, a.pslot);
}

// Host-side launcher shared with the prefill path. `counts` needs nchunks*E ints.
int launch_align_ex(const void* ids, int dt, long N, int k, int E, int BM, int base, int drop, int32_t* st,
                    int32_t* ss, uint8_t* val, int32_t* be, int* counts, cudaStream_t stream, int2* ranges,
                    int32_t* pslot) {
  AlignArgs a;
  a.ranges = ranges;
  a.pslot = pslot;
  a.ids = ids; a.dt = dt; a.M = N * k; a.k = k; a.E = E; a.BM = BM; a.base = base; a.drop = drop;
  a.Pmax = a.M + (long)min(a.M, (long)E) * BM;
  a.nchunks = (int)((a.M + ALIGN_CHUNK - 1) / ALIGN_CHUNK);
  a.st = st; a.ss = ss; a.val = val; a.be = be; a.counts = counts;
  // per-warp count table: 32 warps x E ints; large E runs with fewer threads
  int threads = ALIGN_THREADS;
  while ((size_t)(threads / 32) * E * sizeof(int) > 96 * 1024 && threads > 128) threads /= 2;
  const size_t wc = (size_t)(threads / 32) * E * sizeof(int);
  // The kernels' dynamic shared-memory limit is raised once per device, to what the device's
  // opt-in maximum leaves beside their static arrays, not per call to this call's size: a per-call
  // value could be lowered by a concurrent call with a smaller E between another call's set and
  // its launch, or under a captured graph.
  static int limit_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VQ2_ERR_CUDA;
  if (!limit_set[dev]) {
    int optin = 0;
    cudaFuncAttributes fs, fp;
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncGetAttributes(&fs, align_single_kernel) != cudaSuccess ||
        cudaFuncGetAttributes(&fp, align_place_kernel) != cudaSuccess)
      return VQ2_ERR_CUDA;
    const int lim = optin - (int)max(fs.sharedSizeBytes, fp.sharedSizeBytes);
    if (lim <= 0 ||
        cudaFuncSetAttribute(align_single_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, lim) != cudaSuccess ||
        cudaFuncSetAttribute(align_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, lim) != cudaSuccess)
      return VQ2_ERR_CUDA;
    limit_set[dev] = lim;
  }
  if (wc > (size_t)limit_set[dev]) return VQ2_ERR_SHAPE;
  if (a.nchunks <= 1) {
    align_single_kernel<<<1, threads, wc, stream>>>(a);
  } else {
    align_count_kernel<<<a.nchunks, threads, 0, stream>>>(a);
    align_scan_kernel<<<1, threads, 0, stream>>>(a);
    align_place_kernel<<<a.nchunks, threads, wc, stream>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}

int launch_align(const void* ids, int dt, long N, int k, int E, int BM, int32_t* st, int32_t* ss,
                 uint8_t* val, int32_t* be, int* counts, cudaStream_t stream) {
  return launch_align_ex(ids, dt, N, k, E, BM, 0, 0, st, ss, val, be, counts, stream, nullptr, nullptr);
}

}  // namespace vq2

using namespace vq2;

extern "C" size_t vq2_align_workspace_size(int N, int k, int E) {
  const long M = (long)N * k;
  const long nchunks = (M + ALIGN_CHUNK - 1) / ALIGN_CHUNK;
  return (size_t)(nchunks < 1 ? 1 : nchunks) * E * sizeof(int) + 256;
}

extern "C" int vq2_align(const void* ids, int ids_dtype, int N, int k, int E, int BM, int32_t* st,
                         int32_t* ss, uint8_t* val, int32_t* be, void* ws, size_t ws_bytes, void* stream) {
  if (!ids || !st || !ss || !val || !be) return VQ2_ERR_NULL;
  if (N <= 0 || k <= 0 || E <= 0 || E > ALIGN_MAX_E || BM <= 0) return VQ2_ERR_SHAPE;
  if (ids_dtype != VQ2_ID_I32 && ids_dtype != VQ2_ID_I64) return VQ2_ERR_DTYPE;
  if (!ws || ws_bytes < vq2_align_workspace_size(N, k, E)) return VQ2_ERR_WORKSPACE;
  int* counts = (int*)(((uintptr_t)ws + 255) & ~(uintptr_t)255);
  return launch_align(ids, ids_dtype, N, k, E, BM, st, ss, val, be, counts, (cudaStream_t)stream);
}
