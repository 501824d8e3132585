// K1 — decode MoE for small token batches (replaces vq2_kernel.vq2_moe_fused_10b,
// reference vq2_vllm/kernels/vq2_kernel.py:569-594).
//
// Two persistent kernels, one CTA per SM, chained with programmatic dependent launch:
//   gateup: part[m, s] = (<W_gate,e[i], Hx_n>, <W_up,e[i], Hx_n>) over K-slice s (fp32 scratch)
//   down:   out[n, h] += w_m * <W_down,e[h], H·(silu(sum_s gate) * sum_s up)>  (fp32 red.add)
// for every (token n, slot j) pair m routed to expert e. Every CTA builds the same plan: one unit
// per pair, units ordered by expert (a pair's rank among the pairs ordered by (expert, pair)); the
// flattened (unit, row) space is split evenly over the CTAs.
//
// Per CTA: a producer warp streams contiguous row chunks (lo / hi / scale planes) into a ring
// of shared-memory stages with 1-D bulk async copies (TMA engine, L2 evict-first) and mbarriers;
// 16 consumer warps decode them. Lane l of a warp owns one 64-wide group of a row (a warp covers a
// 32-group K-slice; rows wider than 2048 are split over KH warps): one 16-byte lo load, one 4-byte
// hi load and one fp16 scale per group. A warp decodes one or more rows per pass (independent
// chains) and reduces their partial sums together with a halving shuffle reduction. The 1024x4
// fp16 codebook is replicated 16x in shared memory so that lane l reads only from bank pair
// (l mod 16): a half-warp's 8-byte gathers are conflict-free. The activation of a unit is staged
// once per CTA: each 64-group is rotated by a warp-shuffle FWHT (the Hadamard), scaled by a power
// of two chosen from the group max and the codebook max so that no half2 partial can overflow,
// and stored as half2 in conflict-free padded rows; a group's 16 codebook-vector x activation
// products accumulate in packed half2 FMAs, and groups combine in fp32 with their scales.
#include <cstddef>
#include "vq2_common.cuh"

namespace vq2 {

#ifndef VQ2_DEC_NW
#define VQ2_DEC_NW 16
#endif
constexpr int DEC_NW = VQ2_DEC_NW;        // consumer warps
constexpr int DEC_THREADS = (DEC_NW + 1) * 32;
constexpr int DEC_TT = 1;                 // tokens per unit (a unit = one (expert, token) pair)
#ifndef VQ2_DEC_STAGES
#define VQ2_DEC_STAGES 3
#endif
#ifndef VQ2_DEC_SA
#define VQ2_DEC_SA 8
#endif
#ifndef VQ2_DEC_SB
#define VQ2_DEC_SB 32
#endif
constexpr int DEC_STAGES = VQ2_DEC_STAGES;
constexpr int DEC_GRAN = 8;               // row granule of the work split (keeps copies 16-B sized)
constexpr int DEC_SA = VQ2_DEC_SA;        // gate/up row pairs per stage
constexpr int DEC_SB = VQ2_DEC_SB;        // down rows per stage
constexpr int DEC_MAXG = 64;              // max 64-groups per input row (4096 / 64)
#ifndef VQ2_DEC_CB_COPIES
#define VQ2_DEC_CB_COPIES 16
#endif
constexpr int CB_COPIES = VQ2_DEC_CB_COPIES;     // codebook copies in shared memory (16: 128 KB)
constexpr int CB_SHIFT = CB_COPIES == 16 ? 7 : 6;  // log2(bytes per entry = 8 x copies)
constexpr int CB_BYTES = 1024 * 8 * CB_COPIES;

struct DecodeShared {
  uint64_t full[DEC_STAGES];
  uint64_t empty[DEC_STAGES];
  uint64_t cbbar;
  int nunits;
  int abort;
  int ep_last;                              // expert parallelism: this CTA completed the down grid
  float cmax;
  float red[32];
  float ginv[DEC_MAXG];                     // per 64-group: 2^-scale / 8 of the staged activation
  // rotated, scaled activation of the staged unit(s), half2 per group; rows padded to 36 words so
  // that lane l's 16-byte reads of row (base + l) start at bank 4l mod 32 (conflict-free)
  alignas(16) uint32_t xs[DEC_MAXG][36];
  // prologue: the codebook as loaded (bulk-copy destination, 8 KB); main loop (down kernel): the
  // combined silu(gate) * up row of the current unit, fp32, before rotation
  alignas(16) float scratch[DEC_MAXG * 64];
  short unit_e[VQ2_DECODE_MAX_PAIRS];
  float unit_w[VQ2_DECODE_MAX_PAIRS];       // routing weight of the unit's pair
  short unit_m[VQ2_DECODE_MAX_PAIRS][DEC_TT];
  alignas(16) int ekey[VQ2_DECODE_MAX_PAIRS];
};


// ------------------------------------------------------------------ plan: group pairs by expert
// Unit u = one (local expert, pair) with units ordered by expert and, within an expert, by pair
// index. Pair m's unit is its rank: the number of valid pairs q with (e_q, q) < (e_m, m). Every
// CTA builds the same plan (M <= VQ2_DECODE_MAX_PAIRS, so the O(M) rank scan per pair is short;
// it reads the keys four at a time as shared-memory broadcasts).
static_assert(DEC_TT == 1, "one pair per unit");
__device__ void build_plan(const void* ids, int ids_dtype, const float* topk_w, int M, int E, int expert_base,
                           DecodeShared* sh) {
  const int tid = threadIdx.x;
  static_assert(DEC_THREADS >= VQ2_DECODE_MAX_PAIRS, "build_plan holds one pair per thread");
  const int M4 = (M + 3) & ~3;
  int valid = 0;
  float w = 0.f;
  if (tid < M4) {                               // one pair per thread (blockDim > max pairs)
    int key = 0x7FFFFFFF;                       // padding / foreign expert: sorts last, never counted
    if (tid < M) {
      const int e = load_id(ids, ids_dtype, tid) - expert_base;
      w = topk_w[tid];
      if (e >= 0 && e < E) { key = e; valid = 1; }
    }
    sh->ekey[tid] = key;
  }
  const int nunits = __syncthreads_count(valid);
  if (tid < M && sh->ekey[tid] != 0x7FFFFFFF) {
    const int m = tid, e = sh->ekey[m];
    int rank = 0;
    for (int q = 0; q < M4; q += 4) {
      const int4 k4 = *(const int4*)&sh->ekey[q];
      rank += (k4.x < e || (k4.x == e && q < m)) + (k4.y < e || (k4.y == e && q + 1 < m)) +
              (k4.z < e || (k4.z == e && q + 2 < m)) + (k4.w < e || (k4.w == e && q + 3 < m));
    }
    sh->unit_e[rank] = (short)e;
    sh->unit_m[rank][0] = (short)m;
    sh->unit_w[rank] = w;
  }
  if (tid == 0) sh->nunits = nunits;
  __syncthreads();
}

// ------------------------------------------------------------------ chunk iteration
struct ChunkIter {
  // The CTA's range [r, end) is contiguous, so the (unit, row) position is found by one division
  // here and then advanced incrementally (no 64-bit divide per chunk).
  int u, row0, left;  // current unit, row within it, rows of the range still to hand out
  int rows_per_unit, S;
  // 32-bit arithmetic: total_rows <= max pairs * 4096 rows = 2^21, grid <= 1024 CTAs.
  __device__ ChunkIter(long total_rows, int rpu, int S_) : rows_per_unit(rpu), S(S_) {
    const unsigned ng = (unsigned)total_rows / DEC_GRAN;
    const unsigned r = blockIdx.x * ng / gridDim.x * DEC_GRAN;
    const unsigned end = (blockIdx.x + 1) * ng / gridDim.x * DEC_GRAN;
    u = (int)(r / (unsigned)rpu);
    row0 = (int)(r - (unsigned)u * rpu);
    left = (int)(end - r);
  }
  __device__ bool next(int& uo, int& row0o, int& n) {
    if (left <= 0) return false;
    n = min(S, min(rows_per_unit - row0, left));
    uo = u;
    row0o = row0;
    left -= n;
    row0 += n;
    if (row0 == rows_per_unit) { row0 = 0; ++u; }
    return true;
  }
};


// consumer-only barrier (named barrier 1; the producer warp never joins it)
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"r"(DEC_NW * 32) : "memory");
}

// ------------------------------------------------------------------ fused expert-parallel exchange
// With `world` > 0 the two kernels also carry the decode step's token exchange between the ranks of
// an expert-parallel group (one exchange region per rank, mapped by every peer; field pointers per
// rank in `peers`, EP_FIELDS each): a small push kernel ahead of them stores this rank's rows, ids
// (as i32) and weights into slot `rank` of every rank's region, the gate/up kernel waits (bounded)
// until every rank's have arrived, and the kernels then run on the gathered rows (world x N
// tokens, this rank's experts);
// the down kernel adds its results with fp32 atomics straight into the owning rank's COMB rows over
// NVLink; its last CTA releases a completion flag to every rank, waits for every rank's flag,
// copies this rank's COMB rows out and re-zeroes them. Steps are numbered by EPOCH in the region.
struct DecEp {
  const uint64_t* peers;    // [world][EP_FIELDS] field addresses of every rank's region
  int world, rank, N;       // N: tokens per rank
  int row_x, ids_i64, k;
  const uint8_t* x_local;   // this rank's N rows, ids and weights
  const void* ids_local;
  const float* w_local;
  const unsigned* dflag;    // this rank's DFLAG [world][VQ2_EP_CTAS] and step counter
  unsigned* epoch;
  unsigned* count;          // this rank's completion counter (the down kernel's CTAs)
  const unsigned* cflag;    // this rank's CFLAG [world]
  float* comb;              // this rank's COMB rows [N][H] (summed by every rank's down kernel)
  float* out;               // this rank's result [N][H]
  int H;
  int keep_out;             // (world 0) the output already holds values to add to: do not zero it
};

// Step number of the current call (EPOCH is advanced by the finish kernel of the previous step).
__device__ __forceinline__ unsigned ep_step(const DecEp& ep) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ep.epoch) : "memory");
  return v + 1;
}

// Every thread: wait until all world x C dispatch flags here reached `step`, then a CTA barrier.
__device__ __forceinline__ void ep_wait_dispatch(const DecEp& ep, unsigned step) {
  const int C = ep_slices((size_t)ep.N * ep.row_x);
  for (int f = threadIdx.x; f < ep.world * C; f += blockDim.x) ep_wait_flag(ep.dflag + f, step);
  __syncthreads();
}

// grid: world x C CTAs (C = ep_slices(N * row_x)), launched ahead of the gate/up kernel: CTA
// (p, c) pushes slice c of this rank's rows, ids (as i32) and weights into slot `rank` of rank p's
// region and releases flag [rank][c] there. The kernel is small, so the gate/up kernel (launched
// behind it with programmatic dependent launch) becomes resident while the rows cross NVLink; the
// gate/up kernel then waits for every rank's flags.
__global__ void __launch_bounds__(512) ep_push_kernel(DecEp ep) {
  pdl_wait();                  // the previous step (whose finish kernel precedes) is complete
  pdl_launch_dependents();
  const unsigned step = ep_step(ep);
  const int C = ep_slices((size_t)ep.N * ep.row_x);
  const size_t xb = (size_t)ep.N * ep.row_x, ib = (size_t)ep.N * ep.k * 4;
  {
    const int b = blockIdx.x;
    const int p = b / C, c = b % C;
    size_t xb0, xb1, ib0, ib1;
    ep_slice(xb, c, C, 16, xb0, xb1);
    ep_slice(ib, c, C, 4, ib0, ib1);
    const uint64_t* t = ep.peers + p * EP_FIELDS;
    uint8_t* dx = (uint8_t*)t[EP_X] + ep.rank * xb;
    for (size_t i = xb0 / 16 + threadIdx.x; i < xb1 / 16; i += blockDim.x)
      ((uint4*)dx)[i] = ((const uint4*)ep.x_local)[i];
    int32_t* di = (int32_t*)((uint8_t*)t[EP_IDS] + ep.rank * ib);
    float* dw = (float*)((uint8_t*)t[EP_WT] + ep.rank * ib);
    for (size_t i = ib0 / 4 + threadIdx.x; i < ib1 / 4; i += blockDim.x) {
      di[i] = ep.ids_i64 ? (int32_t)((const long long*)ep.ids_local)[i] : ((const int32_t*)ep.ids_local)[i];
      dw[i] = ep.w_local[i];
    }
    __syncthreads();                     // every thread's stores precede the release below
    if (threadIdx.x == 0) st_release_sys((unsigned*)t[EP_DFLAG] + ep.rank * C + c, step);
  }
}

// Consumer threads, after the down phase: the CTA's atomics are complete. The CTA that completes
// the count releases this rank's completion flag [rank] at every rank, waits (bounded) for every
// rank's flag here, copies this rank's COMB rows to `out`, re-zeroes them and advances EPOCH
// (every CTA of the grid read EPOCH before it counted itself).
__device__ __forceinline__ void ep_release_done(const DecEp& ep, unsigned step, int* last_flag) {
  consumer_sync();
  if (threadIdx.x == 0) {
    __threadfence_system();
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ep.count) : "memory");
    *last_flag = prev == gridDim.x - 1;
    if (*last_flag) {
      *ep.count = 0;
      for (int p = 0; p < ep.world; ++p)
        st_release_sys((unsigned*)ep.peers[p * EP_FIELDS + EP_CFLAG] + ep.rank, step);
    }
  }
  consumer_sync();
  if (!*last_flag) return;
  for (int f = threadIdx.x; f < ep.world; f += DEC_NW * 32) ep_wait_flag(ep.cflag + f, step);
  consumer_sync();
  const int n4 = ep.N * ep.H / 4;
  for (int i = threadIdx.x; i < n4; i += DEC_NW * 32) {
    ((float4*)ep.out)[i] = __ldcg((const float4*)ep.comb + i);
    ((float4*)ep.comb)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  consumer_sync();
  if (threadIdx.x == 0) {
    __threadfence();   // the zeros reach this GPU's L2 (where the peers' atomics land) first
    *ep.epoch = step;
  }
}

// Consumers replicate the codebook (landed in sh->cbstage by one bulk copy) 16x — entry e of
// copy c at byte e*128 + c*8 — and record max |C| into sh->cmax. Ends with a consumer barrier.
__device__ __forceinline__ void fill_codebook(uint8_t* cbs, DecodeShared* sh) {
  const int tid = threadIdx.x;
  mbar_wait(&sh->cbbar, 0);
  const uint2* src = (const uint2*)sh->scratch;
  float m = 0.f;
  // consecutive threads write consecutive 16-byte chunks (conflict-free stores)
  for (int idx = tid; idx < 1024 * (CB_COPIES / 2); idx += DEC_NW * 32) {
    const int e = idx / (CB_COPIES / 2), k = idx % (CB_COPIES / 2);
    const uint2 v = src[e];
    *(uint4*)(cbs + e * (8 * CB_COPIES) + k * 16) = make_uint4(v.x, v.y, v.x, v.y);
    if (k == 0) {
      const float2 a = __half22float2(*(const __half2*)&v.x), b = __half22float2(*(const __half2*)&v.y);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y))));
    }
  }
  m = warp_max(m);
  if ((tid & 31) == 0) sh->red[tid >> 5] = m;
  consumer_sync();
  if (tid == 0) {
    float r = 0.f;
    for (int w = 0; w < DEC_NW; ++w) r = fmaxf(r, sh->red[w]);
    sh->cmax = fmaxf(r, 1e-30f);
  }
  consumer_sync();
}

// R independent 64-group dot products for NT tokens: for each row r, sum over the group's 16
// sub-vectors of <codebook[id_s], x_s>, accumulated in two half2 chains, returned in fp32.
// lo[r]: the 16 index low bytes; hw[r]: the 4 hi bytes; x[t]: 32 half2 regs of the rotated group.

template <int R, int NT>
__device__ __forceinline__ void multi_dot(const uint4* lo, const uint32_t* hw, const uint8_t* cbl_ptr,
                                          const uint32_t (*x)[32], float (*out)[NT]) {
  const uint32_t cbl = smem_u32(cbl_ptr);          // 32-bit shared-window address of this lane's copy
  __half2 a0[R][NT], a1[R][NT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) { a0[r][t] = __float2half2_rn(0.f); a1[r][t] = a0[r][t]; }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    // each id from one byte permute (ids_hi_pairs / id_of)
    uint32_t Lw[R], h02[R], h13[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      Lw[r] = q == 0 ? lo[r].x : q == 1 ? lo[r].y : q == 2 ? lo[r].z : lo[r].w;
      ids_hi_pairs(__byte_perm(hw[r], 0u, 0x4440 + q), h02[r], h13[r]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = 4 * q + j;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const uint32_t id = j == 0 ? id_of<0>(Lw[r], h02[r], h13[r]) : j == 1 ? id_of<1>(Lw[r], h02[r], h13[r])
                          : j == 2 ? id_of<2>(Lw[r], h02[r], h13[r]) : id_of<3>(Lw[r], h02[r], h13[r]);
        const uint2 c = lds64(cbl + (id << CB_SHIFT));
        const __half2 c01 = *(const __half2*)&c.x, c23 = *(const __half2*)&c.y;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          __half2& acc = (s & 1) ? a1[r][t] : a0[r][t];
          acc = __hfma2(c01, *(const __half2*)&x[t][2 * s], acc);
          acc = __hfma2(c23, *(const __half2*)&x[t][2 * s + 1], acc);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float2 f = __half22float2(__hadd2(a0[r][t], a1[r][t]));
      out[r][t] = f.x + f.y;
    }
}

// Sum V (= 1, 2, 4 or 8) per-lane values over the warp with V + 1 shuffles instead of 5V: each
// halving step keeps half of the values per lane. Afterwards every lane holds the total of value
// reduce_index<V>(lane).
template <int V>
__device__ __forceinline__ int reduce_index(int lane) {
  return V == 8 ? (lane >> 2) & 7 : V == 4 ? (lane >> 3) & 3 : V == 2 ? (lane >> 4) & 1 : 0;
}
template <int V>
__device__ __forceinline__ float warp_reduce_multi(float* v) {
  const int lane = threadIdx.x & 31;
  int n = V;
#pragma unroll
  for (int o = 16; o >= 4; o >>= 1) {
    if (n > 1) {
      const bool hi = (lane & o) != 0;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < n / 2) {
          const float send = hi ? v[i] : v[i + n / 2];
          const float keep = hi ? v[i + n / 2] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      n >>= 1;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
    }
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return v[0];
}

// CTA-wide staging of one unit's activation. Consumer warp w rotates the 64-groups g = w, w + NW,
// ... with a shuffle FWHT (lane holds elements lane and lane + 32 of a group; ld(i) reads element i
// of the row as fp32), scales each group by a power of two chosen from the group's max so that
// max|x| * max|C| * 32 <= 2^15 (no half2 partial of the group's dot products can overflow), and
// stores it as half2 in sh->xs[g]; sh->ginv[g] gets the factor undoing the scale and the
// Hadamard's 1/8. Called by all consumer threads.
constexpr int STAGE_GPW = (DEC_MAXG + DEC_NW - 1) / DEC_NW;   // groups per consumer warp

// Load half of the staging: this lane's elements (lane, lane + 32) of the warp's groups.
template <typename LoadF>
__device__ __forceinline__ void stage_load(LoadF ld, int ng, float* va, float* vb) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < STAGE_GPW; ++i) {   // all loads first, so their latencies overlap
    const int g = warp + i * DEC_NW;
    va[i] = vb[i] = 0.f;
    if (g < ng) { va[i] = ld(g * 64 + lane); vb[i] = ld(g * 64 + 32 + lane); }
  }
}

// Rotate-and-store half of the staging (needs sh->cmax; the caller has synchronised the consumers
// since xs / ginv were last read).
__device__ __forceinline__ void stage_rotate(int ng, DecodeShared* sh, const float* va, const float* vb) {
  constexpr int GPW = STAGE_GPW;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float climit = 1024.f / sh->cmax;
#pragma unroll
  for (int i = 0; i < GPW; ++i) {
    // straight-line over the warp's groups (a group past ng rotates zeros and stores nothing), so
    // the groups' shuffle chains interleave
    const int g = warp + i * DEC_NW;
    const bool gok = g < ng;
    {
      float a = va[i], b = vb[i];
      const float t = a + b;
      b = a - b;
      a = t;
#pragma unroll
      for (int len = 16; len >= 1; len >>= 1) {
        const float pa = __shfl_xor_sync(0xffffffffu, a, len), pb = __shfl_xor_sync(0xffffffffu, b, len);
        a = (lane & len) ? (pa - a) : (a + pa);
        b = (lane & len) ? (pb - b) : (b + pb);
      }
      const float gmax = warp_max(fmaxf(fabsf(a), fabsf(b)));
      float sc = 1.f, inv = 1.f;
      if (gmax > 0.f) {
        // s = floor(log2(ratio)) from the exponent field (ratio > 0; subnormal reads as -127,
        // inf as +128, both clamped); 2^s and 2^-s are built from exponent bits (|s| <= 100)
        const float ratio = climit / gmax;
        const int s = max(-100, min(100, (int)((__float_as_uint(ratio) >> 23) & 0xFF) - 127));
        sc = __uint_as_float((uint32_t)(127 + s) << 23);
        inv = __uint_as_float((uint32_t)(127 - s) << 23);
      }
      const float ea = a * sc, eb = b * sc;
      const float na = __shfl_down_sync(0xffffffffu, ea, 1), nb = __shfl_down_sync(0xffffffffu, eb, 1);
      if (gok && !(lane & 1)) {                   // element pairs (2j, 2j+1) -> half2 j
        __half2 h0 = __floats2half2_rn(ea, na), h1 = __floats2half2_rn(eb, nb);
        sh->xs[g][lane >> 1] = *(uint32_t*)&h0;
        sh->xs[g][16 + (lane >> 1)] = *(uint32_t*)&h1;
      }
      if (gok && lane == 0) sh->ginv[g] = inv * 0.125f;
    }
  }
  consumer_sync();
}

template <typename LoadF>
__device__ __forceinline__ void stage_activation(LoadF ld, int ng, DecodeShared* sh) {
  float va[STAGE_GPW], vb[STAGE_GPW];
  consumer_sync();                         // the previous unit's xs / ginv are no longer read
  stage_load(ld, ng, va, vb);
  stage_rotate(ng, sh, va, vb);
}

// A consumer lane's copy of its group's staged activation (zeros past the row's groups).
__device__ __forceinline__ void load_xs(const DecodeShared* sh, int g, bool gv, uint32_t* xr) {
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    const uint4 q = gv ? *(const uint4*)&sh->xs[g][i] : make_uint4(0, 0, 0, 0);
    xr[i] = q.x; xr[i + 1] = q.y; xr[i + 2] = q.z; xr[i + 3] = q.w;
  }
}

// Shared-memory carve-up.
struct DecSmem {
  uint8_t* cbs;
  DecodeShared* sh;
  uint8_t* stages;
};
__device__ __forceinline__ DecSmem dec_smem(uint8_t* smem) {
  DecSmem d;
  d.cbs = smem;
  d.sh = (DecodeShared*)(smem + CB_BYTES);
  d.stages = smem + CB_BYTES + ((sizeof(DecodeShared) + 127) / 128) * 128;
  return d;
}

// Barrier init and codebook bulk copy (thread 0; the codebook is a constant weight, so this may
// run before the grid-dependency wait).
__device__ __forceinline__ void dec_init(const uint16_t* cb, DecSmem d) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < DEC_STAGES; ++s) { mbar_init(&d.sh->full[s], 1); mbar_init(&d.sh->empty[s], DEC_NW); }
    mbar_init(&d.sh->cbbar, 1);
    d.sh->abort = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(&d.sh->cbbar, 1024 * 4 * 2);
    bulk_g2s(d.sh->scratch, cb, 1024 * 4 * 2, &d.sh->cbbar);
  }
}
// Barrier init, codebook bulk copy, expert plan (all threads; ends with __syncthreads).
__device__ __forceinline__ void dec_prologue(const vq2_moe_args& a, const uint16_t* cb, DecSmem d) {
  dec_init(cb, d);
  build_plan(a.topk_ids, a.ids_dtype, a.topk_w, a.N * a.topk, a.E, a.expert_base, d.sh);
}

// One pass of a consumer warp over RB gate/up row pairs of a stage (rows rr0 + k*rstep):
// 2*RB group dot products, one batched reduction, 2*RB writer lanes.
template <int RB>
__device__ __forceinline__ void gateup_rows(const uint8_t* st, int rr0, int rstep, int n, int g, bool gv, int nsub,
                                            int ng, uint32_t lo_b, uint32_t hi_b, uint32_t sc_b, const uint8_t* cbl,
                                            const uint32_t (*xr)[32], float inv, int m, int KH, int h, int I,
                                            int i0, float* part) {
  constexpr int R = 2 * RB;
  uint4 lo[R];
  uint32_t hw[R];
  float sc[R];
#pragma unroll
  for (int k = 0; k < RB; ++k) {
    const int rr = rr0 + k * rstep;
    if (gv && rr < n) {
#pragma unroll
      for (int u = 0; u < 2; ++u) {   // u = 0 gate row, 1 up row
        lo[2 * k + u] = *(const uint4*)(st + u * lo_b + rr * nsub + g * 16);
        hw[2 * k + u] = *(const uint32_t*)(st + 2 * lo_b + u * hi_b + rr * (nsub / 4) + g * 4);
        sc[2 * k + u] = __half2float(*(const __half*)(st + 2 * (lo_b + hi_b) + u * sc_b + (rr * ng + g) * 2));
      }
    } else {
#pragma unroll
      for (int u = 0; u < 2; ++u) { lo[2 * k + u] = make_uint4(0, 0, 0, 0); hw[2 * k + u] = 0; sc[2 * k + u] = 0.f; }
    }
  }
  float d[R][1];
  multi_dot<R, 1>(lo, hw, cbl, xr, d);
  float v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = d[r][0] * sc[r] * inv;
  const float tot = warp_reduce_multi<R>(v);
  const int lane = threadIdx.x & 31;
  const int r = reduce_index<R>(lane);
  const int rr = rr0 + (r >> 1) * rstep;
  if ((lane & (32 / R - 1)) == 0 && rr < n) part[((m * KH + h) * 2 + (r & 1)) * I + i0 + rr] = tot;
}

// One pass of a consumer warp over R down rows of a stage (rows rr0 + r*rstep).
template <int R>
__device__ __forceinline__ void down_rows(const uint8_t* st, int rr0, int rstep, int n, int g, bool gv, int nsub,
                                          int ng, uint32_t lo_b, uint32_t hi_b, const uint8_t* cbl,
                                          const uint32_t (*xr)[32], float wsc, int h0, float* orow) {
  uint4 lo[R];
  uint32_t hw[R];
  float sc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int rr = rr0 + r * rstep;
    if (gv && rr < n) {
      lo[r] = *(const uint4*)(st + rr * nsub + g * 16);
      hw[r] = *(const uint32_t*)(st + lo_b + rr * (nsub / 4) + g * 4);
      sc[r] = __half2float(*(const __half*)(st + lo_b + hi_b + (rr * ng + g) * 2));
    } else {
      lo[r] = make_uint4(0, 0, 0, 0); hw[r] = 0; sc[r] = 0.f;
    }
  }
  float d[R][1];
  multi_dot<R, 1>(lo, hw, cbl, xr, d);
  float v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = d[r][0] * sc[r] * wsc;
  const float tot = warp_reduce_multi<R>(v);
  const int lane = threadIdx.x & 31;
  const int r = reduce_index<R>(lane);
  const int rr = rr0 + r * rstep;
  if ((lane & (32 / R - 1)) == 0 && rr < n) atomicAdd(&orow[h0 + rr], tot);
}

// ------------------------------------------------------------------ phases
// Every kernel's ring slot is DEC_STAGE_BYTES: gate/up stages DEC_SA row pairs of an H-wide
// expert (H <= 4096), down stages down_rows_per_stage(KH) rows of an I-wide one (I <= 4096).
constexpr uint32_t DEC_ROW_BYTES_4K = 4096 / 4 + 4096 / 16 + 4096 / 32;   // lo + hi + scales, 4096 wide
constexpr uint32_t DEC_STAGE_BYTES = DEC_SA * 2 * DEC_ROW_BYTES_4K;
__host__ __device__ constexpr int down_rows_per_stage(int KH) { return DEC_SB / KH; }
static_assert(DEC_SB * DEC_ROW_BYTES_4K / 2 <= DEC_STAGE_BYTES, "down stage (I <= 4096) exceeds the slot");

// Producer (one lane): gate/up row chunks of this CTA's range into the ring, chunk counter c.
__device__ __forceinline__ void gateup_produce(const vq2_moe_args& a, const DecSmem& d, uint64_t pol, int& c) {
  DecodeShared* sh = d.sh;
  const int H = a.H, I = a.I, nsub = H / 4, ng = H / 64;
  constexpr int S = DEC_SA;
  const uint32_t lo_b = S * nsub, hi_b = S * (nsub / 4), sc_b = S * ng * 2;
  ChunkIter it((long)sh->nunits * I, I, S);
  int u, i0, n;
  while (it.next(u, i0, n)) {
    const int slot = c % DEC_STAGES;
    if (c >= DEC_STAGES && !mbar_wait(&sh->empty[slot], ((c / DEC_STAGES) - 1) & 1)) { sh->abort = 1; return; }
    const long e = sh->unit_e[u];
    const long rg = e * 2 * I + i0, ru = rg + I;
    uint8_t* st = d.stages + slot * DEC_STAGE_BYTES;
    mbar_arrive_expect_tx(&sh->full[slot], 2u * n * (nsub + nsub / 4 + ng * 2));
    bulk_g2s_stream(st, a.w13_lo + rg * nsub, n * nsub, &sh->full[slot], pol);
    bulk_g2s_stream(st + lo_b, a.w13_lo + ru * nsub, n * nsub, &sh->full[slot], pol);
    bulk_g2s_stream(st + 2 * lo_b, a.w13_hi + rg * (nsub / 4), n * (nsub / 4), &sh->full[slot], pol);
    bulk_g2s_stream(st + 2 * lo_b + hi_b, a.w13_hi + ru * (nsub / 4), n * (nsub / 4), &sh->full[slot], pol);
    bulk_g2s_stream(st + 2 * (lo_b + hi_b), a.w13_sc + rg * ng, n * ng * 2, &sh->full[slot], pol);
    bulk_g2s_stream(st + 2 * (lo_b + hi_b) + sc_b, a.w13_sc + ru * ng, n * ng * 2, &sh->full[slot], pol);
    ++c;
  }
}

// Producer (one lane): down row chunks. The weights do not depend on the gate/up results.
template <int KH>
__device__ __forceinline__ void down_produce(const vq2_moe_args& a, const DecSmem& d, uint64_t pol, int& c) {
  DecodeShared* sh = d.sh;
  const int H = a.H, I = a.I, nsub = I / 4, ng = I / 64;
  constexpr int S = down_rows_per_stage(KH);
  const uint32_t lo_b = S * nsub, hi_b = S * (nsub / 4);
  ChunkIter it((long)sh->nunits * H, H, S);
  int u, h0, n;
  while (it.next(u, h0, n)) {
    const int slot = c % DEC_STAGES;
    if (c >= DEC_STAGES && !mbar_wait(&sh->empty[slot], ((c / DEC_STAGES) - 1) & 1)) { sh->abort = 1; return; }
    const long r = (long)sh->unit_e[u] * H + h0;
    uint8_t* st = d.stages + slot * DEC_STAGE_BYTES;
    mbar_arrive_expect_tx(&sh->full[slot], (uint32_t)n * (nsub + nsub / 4 + ng * 2));
    bulk_g2s_stream(st, a.w2_lo + r * nsub, n * nsub, &sh->full[slot], pol);
    bulk_g2s_stream(st + lo_b, a.w2_hi + r * (nsub / 4), n * (nsub / 4), &sh->full[slot], pol);
    bulk_g2s_stream(st + lo_b + hi_b, a.w2_sc + r * ng, n * ng * 2, &sh->full[slot], pol);
    ++c;
  }
}

// Producer: every issued copy must land before the CTA exits.
__device__ __forceinline__ void produce_drain(const DecSmem& d, int c) {
  for (int q = max(0, c - DEC_STAGES); q < c; ++q) mbar_wait(&d.sh->full[q % DEC_STAGES], (q / DEC_STAGES) & 1);
}

// Consumers, before the gate/up phase: load the first unit's activation (its latency overlaps the
// codebook fill that follows), zero the output rows the down phase accumulates into.
struct GateupPre {
  float va[STAGE_GPW], vb[STAGE_GPW];
  int m = -1;
};
__device__ __forceinline__ void gateup_pre(const vq2_moe_args& a, const DecSmem& d, GateupPre& pre, bool zero_out) {
  DecodeShared* sh = d.sh;
  const ChunkIter it0((long)sh->nunits * a.I, a.I, DEC_SA);
  if (it0.left > 0) {
    pre.m = sh->unit_m[it0.u][0];
    if (a.N != 1) {   // (one token: its row was loaded before the plan, gateup_load_single)
      const size_t xrow = (size_t)(pre.m / a.topk) * a.H;
      const void* xp = a.x;
      const int xdt = a.x_dtype;
      stage_load([&](int i) { return load_act(xp, xdt, xrow + i); }, a.H / 64, pre.va, pre.vb);
    }
  }
  if (!zero_out) return;
  const long tot = (long)a.N * a.H;
  for (long i = (long)blockIdx.x * DEC_NW * 32 + threadIdx.x; i < tot; i += (long)gridDim.x * DEC_NW * 32)
    a.out[i] = 0.f;
}

// Consumers, one token (N == 1): its row is the first unit's activation whatever the plan says, so
// it is loaded before the plan is built (the two loads' latencies overlap).
__device__ __forceinline__ void gateup_load_single(const vq2_moe_args& a, GateupPre& pre) {
  const void* xp = a.x;
  const int xdt = a.x_dtype;
  stage_load([&](int i) { return load_act(xp, xdt, (size_t)i); }, a.H / 64, pre.va, pre.vb);
}

// Consumers: gate/up K-slice partials of this CTA's rows into `part`. KH = K-slices of the
// H-wide input (H/64 groups, 32 per warp). Needs the gate/up codebook in d.cbs.
template <int KH>
__device__ __forceinline__ void gateup_consume(const vq2_moe_args& a, const DecSmem& d, float* __restrict__ part,
                                               const GateupPre& pre, int& c) {
  DecodeShared* sh = d.sh;
  const int H = a.H, I = a.I, nsub = H / 4, ng = H / 64;
  constexpr int S = DEC_SA;
  const uint32_t lo_b = S * nsub, hi_b = S * (nsub / 4), sc_b = S * ng * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = warp % KH, rsub = warp / KH, rstep = DEC_NW / KH;
  const int g = h * 32 + lane;
  const bool gv = g < ng;
  const uint8_t* cbl = d.cbs + (lane & (CB_COPIES - 1)) * 8;
  uint32_t xr[1][32];
  float inv = 0.f;
  int mcur = -1, ucur = -1;
  ChunkIter it((long)sh->nunits * I, I, S);
  int u, i0, n;
  while (it.next(u, i0, n)) {
    const int slot = c % DEC_STAGES;
    if (u != ucur) {   // uniform across consumer warps: all walk the same chunk list
      ucur = u;
      const int mprev = mcur;
      mcur = sh->unit_m[u][0];
      if (mprev < 0 && mcur == pre.m) {       // first unit: loaded before the codebook fill
        stage_rotate(ng, sh, pre.va, pre.vb);
        load_xs(sh, g, gv, xr[0]);
        inv = gv ? sh->ginv[g] : 0.f;
      } else if (mprev < 0 || mprev / a.topk != mcur / a.topk) {   // same token: xs is still valid
        const size_t xrow = (size_t)(mcur / a.topk) * H;
        const void* xp = a.x;
        const int xdt = a.x_dtype;
        stage_activation([&](int i) { return load_act(xp, xdt, xrow + i); }, ng, sh);
        load_xs(sh, g, gv, xr[0]);
        inv = gv ? sh->ginv[g] : 0.f;
      }
    }
    if (!mbar_wait(&sh->full[slot], (c / DEC_STAGES) & 1)) { ++c; break; }
    const uint8_t* st = d.stages + slot * DEC_STAGE_BYTES;
    if (S / rstep >= 4) {
      for (int rr0 = rsub; rr0 < n; rr0 += 4 * rstep)
        gateup_rows<4>(st, rr0, rstep, n, g, gv, nsub, ng, lo_b, hi_b, sc_b, cbl, xr, inv, mcur, KH, h, I, i0, part);
    } else if (S / rstep >= 2) {
      for (int rr0 = rsub; rr0 < n; rr0 += 2 * rstep)
        gateup_rows<2>(st, rr0, rstep, n, g, gv, nsub, ng, lo_b, hi_b, sc_b, cbl, xr, inv, mcur, KH, h, I, i0, part);
    } else {
      for (int rr0 = rsub; rr0 < n; rr0 += rstep)
        gateup_rows<1>(st, rr0, rstep, n, g, gv, nsub, ng, lo_b, hi_b, sc_b, cbl, xr, inv, mcur, KH, h, I, i0, part);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[slot]);
    ++c;
  }
}

// Consumers: down rows of this CTA's range, combined into a.out with fp32 atomics. KH = K-slices
// of the I-wide input; khA = K-slices of the gate/up partials to sum. Needs the down codebook in
// d.cbs and every CTA's gate/up partials visible.
template <int KH>
__device__ __forceinline__ void down_consume(const vq2_moe_args& a, const DecSmem& d, const float* __restrict__ part,
                                             int khA, const DecEp& ep, int& c) {
  DecodeShared* sh = d.sh;
  const int H = a.H, I = a.I, nsub = I / 4, ng = I / 64;
  constexpr int S = down_rows_per_stage(KH);
  const uint32_t lo_b = S * nsub, hi_b = S * (nsub / 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = warp % KH, rsub = warp / KH, rstep = DEC_NW / KH;
  const int g = h * 32 + lane;
  const bool gv = g < ng;
  const uint8_t* cbl = d.cbs + (lane & (CB_COPIES - 1)) * 8;
  uint32_t xr[1][32];
  float wsc = 0.f;
  float* orow = nullptr;
  int ucur = -1;
  ChunkIter it((long)sh->nunits * H, H, S);
  // Units of this CTA's row range: when all of their activations fit the staging buffer they are
  // staged together before the loop (a range that crosses a unit boundary then pays one staging).
  const int ub = it.u, nu = it.left > 0 ? (it.row0 + it.left - 1) / H + 1 : 0;
  const bool all_at_once = nu * ng <= DEC_MAXG;
  // Combine the K-slice partials of units ub + k0 .. ub + k0 + cnt - 1, apply silu(gate) * up
  // (rows of I floats in scratch) and stage them as groups k * ng + g. All consumer threads.
  auto stage_units = [&](int k0, int cnt) {
    const int q4 = I / 4;
    for (int i4 = threadIdx.x; i4 < cnt * q4; i4 += DEC_NW * 32) {
      const int k = i4 / q4, j4 = i4 - k * q4;
      const int m = sh->unit_m[ub + k0 + k][0];
      const float* p = part + (size_t)m * khA * 2 * I + 4 * j4;
      // L2 loads (__ldcg): the partials were written by other SMs in the previous grid
      float4 G = __ldcg((const float4*)p), U = __ldcg((const float4*)(p + I));
      if (khA > 1) {
        const float4 g2 = __ldcg((const float4*)(p + 2 * I)), u2 = __ldcg((const float4*)(p + 3 * I));
        G.x += g2.x; G.y += g2.y; G.z += g2.z; G.w += g2.w;
        U.x += u2.x; U.y += u2.y; U.z += u2.z; U.w += u2.w;
      }
      float4 r;
      r.x = G.x / (1.f + __expf(-G.x)) * U.x;
      r.y = G.y / (1.f + __expf(-G.y)) * U.y;
      r.z = G.z / (1.f + __expf(-G.z)) * U.z;
      r.w = G.w / (1.f + __expf(-G.w)) * U.w;
      *(float4*)&sh->scratch[4 * i4] = r;
    }
    consumer_sync();
    const float* scr = sh->scratch;
    stage_activation([&](int i) { return scr[i]; }, cnt * ng, sh);
  };
  if (all_at_once && nu > 0) stage_units(0, nu);
  int u, h0, n;
  while (it.next(u, h0, n)) {
    const int slot = c % DEC_STAGES;
    if (u != ucur) {
      ucur = u;
      const int m = sh->unit_m[u][0];
      const int tok = m / a.topk;
      // the token's output row: here, or (expert parallelism) in its owner's COMB over NVLink
      orow = ep.world > 0 ? (float*)ep.peers[(tok / ep.N) * EP_FIELDS + EP_COMB] + (size_t)(tok % ep.N) * H
                          : a.out + (size_t)tok * H;
      int gi = g;                      // this lane's group in the staging buffer
      if (all_at_once) gi += (u - ub) * ng;
      else stage_units(u - ub, 1);
      load_xs(sh, gi, gv, xr[0]);
      wsc = sh->unit_w[u] * (gv ? sh->ginv[gi] : 0.f);
    }
    if (!mbar_wait(&sh->full[slot], (c / DEC_STAGES) & 1)) { ++c; break; }
    const uint8_t* st = d.stages + slot * DEC_STAGE_BYTES;
    if (S / rstep >= 8) {
      for (int rr0 = rsub; rr0 < n; rr0 += 8 * rstep)
        down_rows<8>(st, rr0, rstep, n, g, gv, nsub, ng, lo_b, hi_b, cbl, xr, wsc, h0, orow);
    } else if (S / rstep >= 4) {
      for (int rr0 = rsub; rr0 < n; rr0 += 4 * rstep)
        down_rows<4>(st, rr0, rstep, n, g, gv, nsub, ng, lo_b, hi_b, cbl, xr, wsc, h0, orow);
    } else {
      for (int rr0 = rsub; rr0 < n; rr0 += 2 * rstep) {
        if (rr0 + rstep < n)     // both rows of the pass exist
          down_rows<2>(st, rr0, rstep, n, g, gv, nsub, ng, lo_b, hi_b, cbl, xr, wsc, h0, orow);
        else                     // ragged end of a chunk: one row
          down_rows<1>(st, rr0, rstep, n, g, gv, nsub, ng, lo_b, hi_b, cbl, xr, wsc, h0, orow);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[slot]);
    ++c;
  }
}

// ------------------------------------------------------------------ kernel A: gate/up partials
template <int KH>
__global__ void __launch_bounds__(DEC_THREADS, 1)
decode_gateup_kernel(vq2_moe_args a, float* __restrict__ part, DecEp ep) {
  extern __shared__ __align__(128) uint8_t smem[];
  const DecSmem d = dec_smem(smem);
  // Launched with programmatic dependent launch: the CTA becomes resident, copies the codebook (a
  // constant weight) and replicates it in shared memory while the previous kernel drains.
  // Everything after pdl_wait() reads the call's inputs or writes the workspace and output, which
  // the previous kernel may still be using.
  dec_init(a.w13_cb, d);
  __syncthreads();                              // the barriers are initialised
  if (threadIdx.x >> 5 < DEC_NW) fill_codebook(d.cbs, d.sh);
  // expert parallelism: every rank's rows, ids and weights must have arrived (the plan reads them;
  // their flags order them, and the push kernel ahead starts only after the previous step's
  // finish kernel, which waited for every rank's down kernel, so no grid-dependency wait is
  // needed). Otherwise the call's inputs may come from the previous kernel.
  if (ep.world > 0) ep_wait_dispatch(ep, ep_step(ep));
  else pdl_wait();
  // dependents (the down kernel) may launch now: everything this grid waited for is complete
  pdl_launch_dependents();
  GateupPre pre;
  if (a.N == 1 && threadIdx.x >> 5 < DEC_NW) gateup_load_single(a, pre);
  build_plan(a.topk_ids, a.ids_dtype, a.topk_w, a.N * a.topk, a.E, a.expert_base, d.sh);
  int c = 0;
  if (threadIdx.x >> 5 == DEC_NW) {   // producer warp
    if ((threadIdx.x & 31) == 0) {
      gateup_produce(a, d, l2_evict_first(), c);
      produce_drain(d, c);
    }
    return;
  }
  gateup_pre(a, d, pre, ep.world == 0 && !ep.keep_out);
  gateup_consume<KH>(a, d, part, pre, c);
}

// ------------------------------------------------------------------ kernel B: down + combine
template <int KH>
__global__ void __launch_bounds__(DEC_THREADS, 1)
decode_down_kernel(vq2_moe_args a, const float* __restrict__ part, int khA, DecEp ep) {
  extern __shared__ __align__(128) uint8_t smem[];
  const DecSmem d = dec_smem(smem);
  // the next call's gate/up kernel may launch now: before its own grid-dependency wait it only
  // initialises barriers, copies its codebook and replicates it in its shared memory
  pdl_launch_dependents();
  // expert parallelism: the gathered ids the plan reads were written by the peers (their arrival
  // flags are set by now; the acquire makes the data visible to this CTA)
  const unsigned step = ep.world > 0 ? ep_step(ep) : 0u;
  if (ep.world > 0) ep_wait_dispatch(ep, step);
  dec_prologue(a, a.w2_cb, d);
  int c = 0;
  if (threadIdx.x >> 5 == DEC_NW) {   // producer warp: the weights do not depend on the gate/up grid
    if ((threadIdx.x & 31) == 0) {
      down_produce<KH>(a, d, l2_evict_first(), c);
      produce_drain(d, c);
    }
    return;
  }
  fill_codebook(d.cbs, d.sh);
  pdl_wait();   // the gate/up partials and the zeroed output come from the previous grid
  down_consume<KH>(a, d, part, khA, ep, c);
  if (ep.world > 0) ep_release_done(ep, step, &d.sh->ep_last);
}


static size_t decode_smem_bytes(size_t stage_bytes) {
  return CB_BYTES + ((sizeof(DecodeShared) + 127) / 128) * 128 + (size_t)DEC_STAGES * stage_bytes;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

struct DecodeLaunchCache {
  int nsm = 0;
  bool attr_set = false;
};
static DecodeLaunchCache g_dec_cache[64];

}  // namespace vq2

using namespace vq2;


static int khA_of(int H) { return (H / 64 + 31) / 32; }

extern "C" size_t vq2_decode_workspace_size(int N, int topk, int H, int I) {
  return (size_t)N * topk * khA_of(H) * 2 * I * sizeof(float) + 256;
}

// Validation and the two launches; `ep` (world 0: none) selects the fused expert-parallel exchange.
// ctas > 0 runs the persistent grids on that many CTAs (one per SM) instead of one per SM.
static int decode_launch(const vq2_moe_args* a, void* ws, size_t ws_bytes, void* stream, const DecEp& ep,
                         int ctas = 0) {
  if (!a || !a->x || !a->topk_ids || !a->topk_w || !a->out || !a->w13_cb || !a->w13_lo || !a->w13_hi ||
      !a->w13_sc || !a->w2_cb || !a->w2_lo || !a->w2_hi || !a->w2_sc)
    return VQ2_ERR_NULL;
  if (a->N <= 0 || a->topk <= 0 || a->E <= 0 || a->E > 1024 || a->H % 64 || a->I % 64 || a->H < 64 ||
      a->I < 64 || a->H > 4096 || a->I > 4096)
    return VQ2_ERR_SHAPE;
  if ((long)a->N * a->topk > VQ2_DECODE_MAX_PAIRS) return VQ2_ERR_TOO_MANY_PAIRS;
  if (a->x_dtype < 0 || a->x_dtype > 2 || a->ids_dtype < 0 || a->ids_dtype > 1) return VQ2_ERR_DTYPE;
  const void* ptrs[] = {a->x, a->w13_lo, a->w13_hi, a->w13_sc, a->w2_lo, a->w2_hi, a->w2_sc, a->w13_cb, a->w2_cb};
  for (const void* p : ptrs)
    if (!aligned16(p)) return VQ2_ERR_ALIGN;
  if (!ws || ws_bytes < vq2_decode_workspace_size(a->N, a->topk, a->H, a->I)) return VQ2_ERR_WORKSPACE;
  float* part = (float*)(((uintptr_t)ws + 255) & ~(uintptr_t)255);

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VQ2_ERR_NO_DEVICE;
  DecodeLaunchCache& lc = g_dec_cache[dev];
  const size_t sm = decode_smem_bytes(DEC_STAGE_BYTES);   // every kernel: H, I <= 4096
  if (!lc.attr_set) {
    if (cudaDeviceGetAttribute(&lc.nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return VQ2_ERR_CUDA;
    bool ok = true;
    const void* kernels[] = {(const void*)decode_gateup_kernel<1>, (const void*)decode_gateup_kernel<2>,
                             (const void*)decode_down_kernel<1>,   (const void*)decode_down_kernel<2>};
    for (const void* k : kernels)
      ok &= cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) == cudaSuccess;
    if (!ok) return VQ2_ERR_CUDA;
    lc.attr_set = true;
  }
  const int khA = khA_of(a->H), khB = khA_of(a->I);
  vq2_moe_args args = *a;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas > 0 && ctas < lc.nsm ? ctas : lc.nsm);
  cfg.blockDim = dim3(DEC_THREADS);
  cfg.dynamicSmemBytes = sm;
  cfg.stream = (cudaStream_t)stream;
  void (*ka)(vq2_moe_args, float*, DecEp) = khA == 1 ? decode_gateup_kernel<1> : decode_gateup_kernel<2>;
  void (*kb)(vq2_moe_args, const float*, int, DecEp) = khB == 1 ? decode_down_kernel<1> : decode_down_kernel<2>;
  // both kernels use programmatic dependent launch (each waits for its predecessor with
  // griddepcontrol.wait before touching anything the predecessor may produce or still read)
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, ka, args, part, ep) != cudaSuccess) return VQ2_ERR_CUDA;
  if (cudaLaunchKernelEx(&cfg, kb, args, (const float*)part, khA, ep) != cudaSuccess) return VQ2_ERR_CUDA;
  return VQ2_OK;
}

extern "C" int vq2_decode(const vq2_moe_args* a, void* ws, size_t ws_bytes, void* stream) {
  return decode_launch(a, ws, ws_bytes, stream, DecEp{});
}

// ------------------------------------------------------------------ expert-parallel decode step
extern "C" size_t vq2_ep_decode_workspace_size(int world, int N, int topk, int H, int I) {
  return vq2_decode_workspace_size(world * N, topk, H, I);
}

extern "C" int vq2_ep_decode(const vq2_moe_args* a, const uint64_t* peers, int world, int rank, void* my_region,
                             const vq2_ep_layout* lay, void* ws, size_t ws_bytes, void* stream) {
  if (!a || !peers || !my_region || !lay || !a->x || !a->topk_ids || !a->topk_w || !a->out) return VQ2_ERR_NULL;
  if (world < 1 || world > 64 || rank < 0 || rank >= world || a->N <= 0 || a->topk <= 0) return VQ2_ERR_SHAPE;
  if ((long)world * a->N * a->topk > VQ2_DECODE_MAX_PAIRS) return VQ2_ERR_TOO_MANY_PAIRS;
  if (a->x_dtype < 0 || a->x_dtype > 2 || a->ids_dtype < 0 || a->ids_dtype > 1) return VQ2_ERR_DTYPE;
  const size_t offs[] = {lay->off_x, lay->off_ids, lay->off_w, lay->off_comb, lay->off_dflag, lay->off_cflag,
                         lay->off_epoch, lay->off_count};
  for (size_t o : offs)
    if (o & 15) return VQ2_ERR_ALIGN;
  if (!aligned16(a->x) || !aligned16(a->out) || ((uintptr_t)a->topk_ids & 3) || ((uintptr_t)a->topk_w & 3))
    return VQ2_ERR_ALIGN;
  uint8_t* r = (uint8_t*)my_region;
  const int row_x = a->H * (a->x_dtype == VQ2_DT_F32 ? 4 : 2);
  DecEp ep = {};
  ep.peers = peers;
  ep.world = world;
  ep.rank = rank;
  ep.N = a->N;
  ep.row_x = row_x;
  ep.ids_i64 = a->ids_dtype == VQ2_ID_I64;
  ep.k = a->topk;
  ep.x_local = (const uint8_t*)a->x;
  ep.ids_local = a->topk_ids;
  ep.w_local = a->topk_w;
  ep.dflag = (const unsigned*)(r + lay->off_dflag);
  ep.epoch = (unsigned*)(r + lay->off_epoch);
  ep.count = (unsigned*)(r + lay->off_count);
  ep.cflag = (const unsigned*)(r + lay->off_cflag);
  ep.comb = (float*)(r + lay->off_comb);
  ep.out = a->out;
  ep.H = a->H;
  {
    cudaLaunchConfig_t pc = {};
    pc.gridDim = dim3(world * ep_slices((size_t)a->N * row_x));
    pc.blockDim = dim3(512);
    pc.stream = (cudaStream_t)stream;
    cudaLaunchAttribute pa[1];
    pa[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pa[0].val.programmaticStreamSerializationAllowed = 1;
    pc.attrs = pa;
    pc.numAttrs = 1;
    if (cudaLaunchKernelEx(&pc, ep_push_kernel, ep) != cudaSuccess) return VQ2_ERR_CUDA;
  }
  // the kernels run on the gathered rows of all ranks (region fields, i32 ids)
  vq2_moe_args g = *a;
  g.N = world * a->N;
  g.x = r + lay->off_x;
  g.topk_ids = r + lay->off_ids;
  g.ids_dtype = VQ2_ID_I32;
  g.topk_w = (const float*)(r + lay->off_w);
  g.out = (float*)(r + lay->off_comb);   // not written: results go to the owners' COMB rows
  return decode_launch(&g, ws, ws_bytes, stream, ep);
}
// ------------------------------------------------------------------ decode from host buffers
// One call per decode step for a caller whose inputs and result live in host memory: the three
// input copies, both kernels and the output copy are queued on `stream` from C, so a step costs
// one library call on the host. Device staging (caller-owned) holds x | ids | w | out.
static size_t stage_part(size_t b) { return (b + 255) & ~(size_t)255; }

extern "C" size_t vq2_decode_host_stage_size(int N, int topk, int H, int x_dtype, int ids_dtype) {
  if (N <= 0 || topk <= 0 || H <= 0) return 0;
  const size_t xe = x_dtype == VQ2_DT_F32 ? 4 : 2, ie = ids_dtype == VQ2_ID_I64 ? 8 : 4;
  return stage_part((size_t)N * H * xe) + stage_part((size_t)N * topk * ie) + stage_part((size_t)N * topk * 4) +
         stage_part((size_t)N * H * 4) + 256;
}

extern "C" int vq2_decode_host(const vq2_moe_args* a, const void* h_x, const void* h_ids, const float* h_w,
                               float* h_out, void* stage, size_t stage_bytes, void* ws, size_t ws_bytes,
                               void* stream) {
  if (!a || !h_x || !h_ids || !h_w || !h_out || !stage) return VQ2_ERR_NULL;
  if (a->N <= 0 || a->topk <= 0 || a->H <= 0) return VQ2_ERR_SHAPE;
  if (a->x_dtype < 0 || a->x_dtype > 2 || a->ids_dtype < 0 || a->ids_dtype > 1) return VQ2_ERR_DTYPE;
  if (stage_bytes < vq2_decode_host_stage_size(a->N, a->topk, a->H, a->x_dtype, a->ids_dtype))
    return VQ2_ERR_WORKSPACE;
  const size_t xb = (size_t)a->N * a->H * (a->x_dtype == VQ2_DT_F32 ? 4 : 2);
  const size_t ib = (size_t)a->N * a->topk * (a->ids_dtype == VQ2_ID_I64 ? 8 : 4);
  const size_t wb = (size_t)a->N * a->topk * 4, ob = (size_t)a->N * a->H * 4;
  uint8_t* d = (uint8_t*)(((uintptr_t)stage + 255) & ~(uintptr_t)255);
  vq2_moe_args b = *a;
  b.x = d;
  b.topk_ids = d + stage_part(xb);
  b.topk_w = (const float*)(d + stage_part(xb) + stage_part(ib));
  b.out = (float*)(d + stage_part(xb) + stage_part(ib) + stage_part(wb));
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemcpyAsync((void*)b.x, h_x, xb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync((void*)b.topk_ids, h_ids, ib, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync((void*)b.topk_w, h_w, wb, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return VQ2_ERR_CUDA;
  const int rc = vq2_decode(&b, ws, ws_bytes, stream);
  if (rc) return rc;
  return cudaMemcpyAsync(h_out, b.out, ob, cudaMemcpyDeviceToHost, st) == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}

// Pipelined variant for serving loops: the packed inputs (x | ids | w, at the offsets of
// vq2_decode_host_offsets) are uploaded on `in_stream`, the kernels run on `stream` after the
// upload (ev_in), and the result is downloaded on `out_stream` after the kernels (ev_done, then
// ev_out marks the download), so the copies of neighbouring steps overlap this step's kernels.
extern "C" void vq2_decode_host_offsets(int N, int topk, int H, int x_dtype, int ids_dtype, size_t* off_ids,
                                        size_t* off_w, size_t* in_bytes) {
  const size_t xb = (size_t)N * H * (x_dtype == VQ2_DT_F32 ? 4 : 2);
  const size_t ib = (size_t)N * topk * (ids_dtype == VQ2_ID_I64 ? 8 : 4);
  const size_t wb = (size_t)N * topk * 4;
  *off_ids = stage_part(xb);
  *off_w = stage_part(xb) + stage_part(ib);
  *in_bytes = stage_part(xb) + stage_part(ib) + stage_part(wb);
}

extern "C" int vq2_decode_host_async(const vq2_moe_args* a, const void* h_in, float* h_out, void* d_in,
                                     float* d_out, void* ws, size_t ws_bytes, void* stream, void* in_stream,
                                     void* out_stream, void* ev_in, void* ev_done, void* ev_out) {
  if (!a || !h_in || !h_out || !d_in || !d_out || !ev_in || !ev_done || !ev_out) return VQ2_ERR_NULL;
  if (a->N <= 0 || a->topk <= 0 || a->H <= 0) return VQ2_ERR_SHAPE;
  if (a->x_dtype < 0 || a->x_dtype > 2 || a->ids_dtype < 0 || a->ids_dtype > 1) return VQ2_ERR_DTYPE;
  if (((uintptr_t)d_in & 255) != 0) return VQ2_ERR_ALIGN;
  size_t off_i = 0, off_w = 0, nin = 0;
  vq2_decode_host_offsets(a->N, a->topk, a->H, a->x_dtype, a->ids_dtype, &off_i, &off_w, &nin);
  vq2_moe_args b = *a;
  b.x = d_in;
  b.topk_ids = (const uint8_t*)d_in + off_i;
  b.topk_w = (const float*)((const uint8_t*)d_in + off_w);
  b.out = d_out;
  cudaStream_t s = (cudaStream_t)stream, si = (cudaStream_t)in_stream, so = (cudaStream_t)out_stream;
  cudaEvent_t ei = (cudaEvent_t)ev_in, ed = (cudaEvent_t)ev_done, eo = (cudaEvent_t)ev_out;
  // the events still mark this slot's previous step: its kernels must be done with d_in before
  // the upload, and its download done with d_out before the kernels write it
  if (cudaStreamWaitEvent(si, ed, 0) != cudaSuccess ||
      cudaMemcpyAsync(d_in, h_in, nin, cudaMemcpyHostToDevice, si) != cudaSuccess ||
      cudaEventRecord(ei, si) != cudaSuccess || cudaStreamWaitEvent(s, ei, 0) != cudaSuccess ||
      cudaStreamWaitEvent(s, eo, 0) != cudaSuccess)
    return VQ2_ERR_CUDA;
  const int rc = vq2_decode(&b, ws, ws_bytes, stream);
  if (rc) return rc;
  if (cudaEventRecord(ed, s) != cudaSuccess || cudaStreamWaitEvent(so, ed, 0) != cudaSuccess ||
      cudaMemcpyAsync(h_out, d_out, (size_t)a->N * a->H * sizeof(float), cudaMemcpyDeviceToHost, so) != cudaSuccess ||
      cudaEventRecord(eo, so) != cudaSuccess)
    return VQ2_ERR_CUDA;
  return VQ2_OK;
}

static_assert(offsetof(vq2::DecodeShared, xs) % 16 == 0, "xs must be 16-byte aligned");
static_assert(offsetof(vq2::DecodeShared, scratch) % 16 == 0, "bulk-copy destination must be 16-byte aligned");
static_assert(offsetof(vq2::DecodeShared, ekey) % 16 == 0, "ekey is read as int4");

// ------------------------------------------------------------------ allocation-free decode
// For callers that cannot allocate device memory at call time — for example code running under a
// memory pool that forbids new allocations, inside a driver callback, or in a host runtime that
// has no CUDA allocator of its own — this variant takes its gate/up scratch from a fixed array
// compiled into the library instead of a caller workspace. Every GPU that loads the library keeps
// VQ2_NOALLOC_SCRATCH_BYTES reserved for it until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[VQ2_NOALLOC_SCRATCH_BYTES];
static void* g_noalloc_ptr[64];   // device address of the array, looked up once per device

extern "C" int vq2_decode_noalloc(const vq2_moe_args* a, void* stream) {
  if (!a) return VQ2_ERR_NULL;
  if (a->N <= 0 || a->topk <= 0 || a->H <= 0 || a->I <= 0) return VQ2_ERR_SHAPE;
  // the scratch this call needs: fp32 gate/up partials per (pair, K-slice)
  const size_t need = vq2_decode_workspace_size(a->N, a->topk, a->H, a->I) - 256;
  if (need > (size_t)VQ2_NOALLOC_SCRATCH_BYTES) return VQ2_ERR_NOALLOC_LIMIT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VQ2_ERR_NO_DEVICE;
  if (!g_noalloc_ptr[dev]) {
    // The array's host-side name is not a device address; ask the runtime for this device's.
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return VQ2_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  // The partials are fully rewritten before they are read, so nothing needs clearing; the
  // 256-aligned array start means the workspace's alignment slack is not used.
  return vq2_decode(a, g_noalloc_ptr[dev], vq2_decode_workspace_size(a->N, a->topk, a->H, a->I), stream);
}
