// K5 — VQ packer: quantise weight matrices into the vq2 format on the GPU (offline, not on the
// serving path). Replaces the k-means packer of the reference, vq2_kernel.pack_vq2
// (vq2_vllm/kernels/vq2_kernel.py:37-72), whose steps are
//   Wg  = W @ H64 per 64-column group (zero-padded to a group multiple)
//   s   = max(|Wg| over the group, 1e-8);  Wn = Wg / s, viewed as 4-wide sub-vectors
//   C   = k samples of a random sample of Wn; `iters` Lloyd iterations over that sample
//         (nearest centroid, then each non-empty centroid = mean of its members)
//   idx = nearest centroid of every sub-vector;  dq = (C[idx] * s) @ H64^T  (the reconstruction)
//
// Three kernels, each fully defined arithmetic so that results are reproducible bit for bit:
//   gather   one warp per requested sub-vector: rotates its group (the fp32 butterfly of the
//            activation transform) and writes the 4 normalised values.
//   kmeans   per Lloyd iteration an assign+accumulate kernel (one sample per thread, centroids in
//            shared memory) and an update kernel. Member sums are fixed-point int64 (value x 2^40,
//            rounded to nearest even) accumulated with integer atomics, so the order of the
//            additions does not matter; mean = (double)sum * 2^-40 / count, rounded to fp32.
//   assign   each warp takes 8 consecutive groups (128 sub-vectors, flat over rows x groups):
//            rotates and normalises them into shared memory, every lane finds the nearest
//            centroid of 4 consecutive sub-vectors (two per packed f32x2 instruction), and
//            writes the lo plane (one word), the hi byte, the int16 ids, the group scales and,
//            when asked, dq (C[id] * s through the same butterfly, which is its own inverse up
//            to the 1/8 normalisation).
// Distances are ((d0^2 + d1^2) + d2^2) + d3^2 with d = x - c, each operation rounded separately
// (no contraction); the lowest index wins a tie. The reference uses torch.cdist, whose rounding
// differs, so near-ties can resolve differently there.
#include "vq2_common.cuh"

namespace vq2 {

constexpr int PK_MAX_K = 1024;
constexpr int PK_THREADS = 256;
constexpr int PK_GROUPS_PER_WARP = 8;              // 128 sub-vectors, 4 per lane
constexpr float PK_FIX = 1099511627776.0f;         // 2^40
constexpr long long PK_MAX_SAMPLES = 1LL << 23;    // k-means sample limit: 2^23 x 2^40 < 2^63

// Normalised group `gid` (flat over rows x groups) of W [rows][D]: lane holds columns lane and
// lane + 32 of the rotated, normalised group; returns the group scale.
__device__ __forceinline__ float pk_rotate(const void* W, int dt, long long gid, int ng, int D, int lane, float& a,
                                           float& b) {
  const long long row = gid / ng;
  const int g = (int)(gid - row * ng);
  const int c0 = g * 64 + lane, c1 = c0 + 32;
  const size_t base = (size_t)row * D;
  a = c0 < D ? load_act(W, dt, base + c0) : 0.f;
  b = c1 < D ? load_act(W, dt, base + c1) : 0.f;
  float t = a + b;
  b = a - b;
  a = t;
#pragma unroll
  for (int len = 16; len >= 1; len >>= 1) {
    const float pa = __shfl_xor_sync(0xffffffffu, a, len), pb = __shfl_xor_sync(0xffffffffu, b, len);
    a = (lane & len) ? (pa - a) : (a + pa);
    b = (lane & len) ? (pb - b) : (b + pb);
  }
  a *= 0.125f;
  b *= 0.125f;
  const float s = fmaxf(warp_max(fmaxf(fabsf(a), fabsf(b))), 1e-8f);
  a = __fdiv_rn(a, s);
  b = __fdiv_rn(b, s);
  return s;
}

__device__ __forceinline__ float pk_dist(float4 x, float4 c) {
  const float d0 = __fsub_rn(x.x, c.x), d1 = __fsub_rn(x.y, c.y), d2 = __fsub_rn(x.z, c.z), d3 = __fsub_rn(x.w, c.w);
  float s = __fadd_rn(__fmul_rn(d0, d0), __fmul_rn(d1, d1));
  s = __fadd_rn(s, __fmul_rn(d2, d2));
  return __fadd_rn(s, __fmul_rn(d3, d3));
}

__device__ __forceinline__ void pk_load_codebook(float4* cs, const float4* C, int k) {
  for (int c = threadIdx.x; c < k; c += blockDim.x) cs[c] = C[c];
  __syncthreads();
}

__global__ void __launch_bounds__(PK_THREADS) pack_gather_kernel(const void* __restrict__ W, int dt, int D, int ng,
                                                                 const long long* __restrict__ vidx, long long n,
                                                                 long long nvec, float4* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long s = ((long long)blockIdx.x * PK_THREADS + threadIdx.x) >> 5;
  if (s >= n) return;
  const long long v = vidx[s];
  if (v < 0 || v >= nvec) {                 // out-of-range index: skip the load, record the error
    if (lane == 0) set_status(VQ2_ERR_SHAPE);
    return;
  }
  const int j = (int)(v & 15);
  float a, b;
  pk_rotate(W, dt, v >> 4, ng, D, lane, a, b);
  const float src = j < 8 ? a : b;
  const int l0 = 4 * (j & 7);
  float4 r;
  r.x = __shfl_sync(0xffffffffu, src, l0);
  r.y = __shfl_sync(0xffffffffu, src, l0 + 1);
  r.z = __shfl_sync(0xffffffffu, src, l0 + 2);
  r.w = __shfl_sync(0xffffffffu, src, l0 + 3);
  if (lane == 0) out[s] = r;
}

__global__ void __launch_bounds__(PK_THREADS) kmeans_accum_kernel(const float4* __restrict__ samp, long long n,
                                                                  const float4* __restrict__ C, int k,
                                                                  unsigned long long* __restrict__ sums,
                                                                  unsigned int* __restrict__ cnt) {
  __shared__ float4 cs[PK_MAX_K];
  pk_load_codebook(cs, C, k);
  const long long i = (long long)blockIdx.x * PK_THREADS + threadIdx.x;
  if (i >= n) return;
  const float4 x = samp[i];
  float best = INFINITY;
  int bi = 0;
  for (int c = 0; c < k; ++c) {
    const float d = pk_dist(x, cs[c]);
    if (d < best) { best = d; bi = c; }
  }
  atomicAdd(&sums[4 * bi + 0], (unsigned long long)__float2ll_rn(x.x * PK_FIX));
  atomicAdd(&sums[4 * bi + 1], (unsigned long long)__float2ll_rn(x.y * PK_FIX));
  atomicAdd(&sums[4 * bi + 2], (unsigned long long)__float2ll_rn(x.z * PK_FIX));
  atomicAdd(&sums[4 * bi + 3], (unsigned long long)__float2ll_rn(x.w * PK_FIX));
  atomicAdd(&cnt[bi], 1u);
}

// C[c] = mean of its members where it has any; clears the accumulators for the next iteration.
__global__ void kmeans_update_kernel(float* __restrict__ C, int k, unsigned long long* __restrict__ sums,
                                     unsigned int* __restrict__ cnt) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= k) return;
  const unsigned int m = cnt[c];
  if (m) {
#pragma unroll
    for (int d = 0; d < 4; ++d) {
      const double s = __ll2double_rn((long long)sums[4 * c + d]) * 9.094947017729282379150390625e-13;   // 2^-40
      C[4 * c + d] = __double2float_rn(__ddiv_rn(s, (double)m));
    }
  }
#pragma unroll
  for (int d = 0; d < 4; ++d) sums[4 * c + d] = 0ull;
  cnt[c] = 0u;
}

// Two sub-vectors per packed fp32x2 instruction (Blackwell add/sub/mul.rn.f32x2: each half
// rounded to nearest on its own, so the result equals the scalar sequence bit for bit).
__device__ __forceinline__ unsigned long long f2pack(float lo, float hi) {
  unsigned long long d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ void f2unpack(unsigned long long v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long f2sub(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2mul(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ unsigned long long f2add(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Shared memory of the assign kernel: the codebook with every component doubled, centroid c as
// {x, x, y, y}, {z, z, w, w} (so one 16-byte load gives two packed operands), then the per-warp
// staging of 8 rotated groups and their scales.
constexpr size_t PK_ASSIGN_SMEM = (size_t)PK_MAX_K * 32 + (size_t)(PK_THREADS / 32) * PK_GROUPS_PER_WARP * 64 * 4 +
                                  (size_t)(PK_THREADS / 32) * PK_GROUPS_PER_WARP * 4;

__global__ void __launch_bounds__(PK_THREADS) pack_assign_kernel(const void* __restrict__ W, int dt, int D, int ng,
                                                                 long long ngroups, const float4* __restrict__ C,
                                                                 int k, uint8_t* __restrict__ lo,
                                                                 uint8_t* __restrict__ hi, int16_t* __restrict__ idx,
                                                                 float* __restrict__ scale, float* __restrict__ dq) {
  extern __shared__ __align__(16) unsigned char pk_smem[];
  ulonglong2* cs2 = reinterpret_cast<ulonglong2*>(pk_smem);                       // [k][2]
  float (*stage)[PK_GROUPS_PER_WARP * 64] =
      reinterpret_cast<float (*)[PK_GROUPS_PER_WARP * 64]>(pk_smem + (size_t)PK_MAX_K * 32);
  float (*gsc)[PK_GROUPS_PER_WARP] = reinterpret_cast<float (*)[PK_GROUPS_PER_WARP]>(
      pk_smem + (size_t)PK_MAX_K * 32 + (size_t)(PK_THREADS / 32) * PK_GROUPS_PER_WARP * 64 * 4);
  for (int c = threadIdx.x; c < k; c += blockDim.x) {
    const float4 v = C[c];
    cs2[2 * c] = make_ulonglong2(f2pack(v.x, v.x), f2pack(v.y, v.y));
    cs2[2 * c + 1] = make_ulonglong2(f2pack(v.z, v.z), f2pack(v.w, v.w));
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* st = stage[warp];
  const long long ntiles = (ngroups + PK_GROUPS_PER_WARP - 1) / PK_GROUPS_PER_WARP;
  const long long nwarps = (long long)gridDim.x * (PK_THREADS / 32);
  for (long long t = (long long)blockIdx.x * (PK_THREADS / 32) + warp; t < ntiles; t += nwarps) {
    const long long g0 = t * PK_GROUPS_PER_WARP;
#pragma unroll 1
    for (int q = 0; q < PK_GROUPS_PER_WARP; ++q) {
      float a = 0.f, b = 0.f, s = 1.f;
      if (g0 + q < ngroups) s = pk_rotate(W, dt, g0 + q, ng, D, lane, a, b);
      st[q * 64 + lane] = a;
      st[q * 64 + 32 + lane] = b;
      if (lane == 0) gsc[warp][q] = s;
    }
    __syncwarp();
    // lane owns sub-vectors 4*lane .. 4*lane+3 of the tile: floats 16*lane .. 16*lane+15;
    // packed as pairs (0, 1) and (2, 3), one 64-bit register per component
    float4 x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = *reinterpret_cast<const float4*>(st + 16 * lane + 4 * i);
    unsigned long long X[2][4];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      X[p][0] = f2pack(x[2 * p].x, x[2 * p + 1].x);
      X[p][1] = f2pack(x[2 * p].y, x[2 * p + 1].y);
      X[p][2] = f2pack(x[2 * p].z, x[2 * p + 1].z);
      X[p][3] = f2pack(x[2 * p].w, x[2 * p + 1].w);
    }
    float best[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
    int bi[4] = {0, 0, 0, 0};
#pragma unroll 4
    for (int c = 0; c < k; ++c) {
      const ulonglong2 A = cs2[2 * c], B = cs2[2 * c + 1];
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const unsigned long long d0 = f2sub(X[p][0], A.x), d1 = f2sub(X[p][1], A.y);
        const unsigned long long d2 = f2sub(X[p][2], B.x), d3 = f2sub(X[p][3], B.y);
        unsigned long long sacc = f2add(f2mul(d0, d0), f2mul(d1, d1));
        sacc = f2add(sacc, f2mul(d2, d2));
        sacc = f2add(sacc, f2mul(d3, d3));
        float s0, s1;
        f2unpack(sacc, s0, s1);
        if (s0 < best[2 * p]) { best[2 * p] = s0; bi[2 * p] = c; }
        if (s1 < best[2 * p + 1]) { best[2 * p + 1] = s1; bi[2 * p + 1] = c; }
      }
    }
    const int q = lane >> 2;                       // this lane's group within the tile
    const bool ok = g0 + q < ngroups;
    const long long v0 = t * 128 + 4 * lane;       // flat index of the lane's first sub-vector
    if (ok) {
      if (lo) {
        *reinterpret_cast<uint32_t*>(lo + v0) =
            (uint32_t)(bi[0] & 255) | (uint32_t)(bi[1] & 255) << 8 | (uint32_t)(bi[2] & 255) << 16 |
            (uint32_t)(bi[3] & 255) << 24;
        hi[v0 >> 2] = (uint8_t)((bi[0] >> 8) | (bi[1] >> 8) << 2 | (bi[2] >> 8) << 4 | (bi[3] >> 8) << 6);
      }
      if (idx) {
        *reinterpret_cast<uint2*>(idx + v0) =
            make_uint2((uint32_t)bi[0] | (uint32_t)bi[1] << 16, (uint32_t)bi[2] | (uint32_t)bi[3] << 16);
      }
      if ((lane & 3) == 0) scale[g0 + q] = gsc[warp][q];
    }
    if (dq) {
      const float s = gsc[warp][q];
      __syncwarp();
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 cv = C[bi[i]];
        *reinterpret_cast<float4*>(st + 16 * lane + 4 * i) =
            make_float4(__fmul_rn(cv.x, s), __fmul_rn(cv.y, s), __fmul_rn(cv.z, s), __fmul_rn(cv.w, s));
      }
      __syncwarp();
#pragma unroll 1
      for (int qq = 0; qq < PK_GROUPS_PER_WARP; ++qq) {
        const long long gid = g0 + qq;
        if (gid >= ngroups) break;
        float a = st[qq * 64 + lane], b = st[qq * 64 + 32 + lane];
        float tt = a + b;
        b = a - b;
        a = tt;
#pragma unroll
        for (int len = 16; len >= 1; len >>= 1) {
          const float pa = __shfl_xor_sync(0xffffffffu, a, len), pb = __shfl_xor_sync(0xffffffffu, b, len);
          a = (lane & len) ? (pa - a) : (a + pa);
          b = (lane & len) ? (pb - b) : (b + pb);
        }
        const long long row = gid / ng;
        const int c0 = (int)(gid - row * ng) * 64 + lane;
        if (c0 < D) dq[(size_t)row * D + c0] = a * 0.125f;
        if (c0 + 32 < D) dq[(size_t)row * D + c0 + 32] = b * 0.125f;
      }
    }
    __syncwarp();
  }
}

inline int pk_grid(long long warps_needed) {
  long long b = (warps_needed + PK_THREADS / 32 - 1) / (PK_THREADS / 32);
  const long long nsm = std::max(device_sm_count(), 1);
  return (int)std::min<long long>(std::max<long long>(b, 1), nsm * 8);
}

}  // namespace vq2

using namespace vq2;

extern "C" int vq2_pack_gather(const void* W, int w_dtype, long long rows, int D, const long long* vec_idx,
                               long long n, float* out, void* stream) {
  if (!W || !vec_idx || !out) return VQ2_ERR_NULL;
  if (rows <= 0 || D <= 0 || n < 0) return VQ2_ERR_SHAPE;
  if (w_dtype < 0 || w_dtype > 2) return VQ2_ERR_DTYPE;
  if ((uintptr_t)out % 16) return VQ2_ERR_ALIGN;
  if (n == 0) return VQ2_OK;
  const int ng = (D + 63) / 64;
  const long long blocks = (n * 32 + PK_THREADS - 1) / PK_THREADS;
  pack_gather_kernel<<<(unsigned)blocks, PK_THREADS, 0, (cudaStream_t)stream>>>(W, w_dtype, D, ng, vec_idx, n,
                                                                                rows * ng * 16, (float4*)out);
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}

extern "C" size_t vq2_kmeans_workspace_size(int k) {
  if (k <= 0 || k > PK_MAX_K) return 0;
  return (size_t)k * (4 * sizeof(unsigned long long) + sizeof(unsigned int)) + 256;
}

extern "C" int vq2_kmeans(const float* samp, long long n, float* C, int k, int iters, void* ws, size_t ws_bytes,
                          void* stream) {
  if (!samp || !C) return VQ2_ERR_NULL;
  if (n <= 0 || k <= 0 || k > PK_MAX_K || iters < 0) return VQ2_ERR_SHAPE;
  // int64 fixed-point member sums (|value| <= 1, x 2^40) cannot overflow below 2^23 members
  if (n > PK_MAX_SAMPLES) return VQ2_ERR_SHAPE;
  if ((uintptr_t)samp % 16 || (uintptr_t)C % 16) return VQ2_ERR_ALIGN;
  if (!ws || ws_bytes < vq2_kmeans_workspace_size(k)) return VQ2_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned long long* sums = (unsigned long long*)(((uintptr_t)ws + 255) & ~(uintptr_t)255);
  unsigned int* cnt = (unsigned int*)(sums + 4 * (size_t)k);
  if (cudaMemsetAsync(sums, 0, (size_t)k * (4 * sizeof(unsigned long long) + sizeof(unsigned int)), st) != cudaSuccess)
    return VQ2_ERR_CUDA;
  const long long blocks = (n + PK_THREADS - 1) / PK_THREADS;
  for (int it = 0; it < iters; ++it) {
    kmeans_accum_kernel<<<(unsigned)blocks, PK_THREADS, 0, st>>>((const float4*)samp, n, (const float4*)C, k, sums, cnt);
    kmeans_update_kernel<<<(k + 255) / 256, 256, 0, st>>>(C, k, sums, cnt);
  }
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}

extern "C" int vq2_pack_assign(const void* W, int w_dtype, long long rows, int D, const float* C, int k,
                               uint8_t* lo, uint8_t* hi, int16_t* idx, float* scale, float* dq, void* stream) {
  if (!W || !C || !scale || (!lo) != (!hi)) return VQ2_ERR_NULL;
  if (rows <= 0 || D <= 0 || k <= 0 || k > PK_MAX_K) return VQ2_ERR_SHAPE;
  if (w_dtype < 0 || w_dtype > 2) return VQ2_ERR_DTYPE;
  if ((uintptr_t)C % 16 || (uintptr_t)lo % 4 || (uintptr_t)idx % 8 || (uintptr_t)scale % 4 || (uintptr_t)dq % 4)
    return VQ2_ERR_ALIGN;
  const int ng = (D + 63) / 64;
  const long long ngroups = rows * ng;
  const long long tiles = (ngroups + PK_GROUPS_PER_WARP - 1) / PK_GROUPS_PER_WARP;
  if (cudaFuncSetAttribute(pack_assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PK_ASSIGN_SMEM) !=
      cudaSuccess)
    return VQ2_ERR_CUDA;
  pack_assign_kernel<<<pk_grid(tiles), PK_THREADS, PK_ASSIGN_SMEM, (cudaStream_t)stream>>>(W, w_dtype, D, ng, ngroups,
                                                                              (const float4*)C, k, lo, hi, idx,
                                                                              scale, dq);
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}
