// K1 — decode MoE for small token batches (replaces vq2_kernel.vq2_moe_fused_10b,
// reference vq2_vllm/kernels/vq2_kernel.py:569-594).
//
// Two persistent kernels, one CTA per SM, chained with programmatic dependent launch:
//   gateup: inter[m, i] = silu(<W_gate,e[i], Hx_n>) * <W_up,e[i], Hx_n>       (fp32 scratch)
//   down:   out[n, h]  += w_m * <W_down,e[h], H·inter[m]>                       (fp32 red.add)
// for every (token n, slot j) pair m routed to expert e. Pairs are grouped by expert so each
// expert's index planes stream from HBM once per group of up to TT tokens.
//
// Per CTA: a producer warp streams contiguous row chunks (lo / hi / scale planes) into a ring
// of shared-memory stages with 1-D bulk async copies (TMA engine) and mbarriers; consumer warps
// decode them. Lane l of a warp owns the 64-wide groups l, l+32 of a row: one 16-byte lo load,
// one 4-byte hi load and one fp16 scale per group. The 1024x4 fp16 codebook is replicated 16x
// in shared memory so that lane l reads only from bank pair (l mod 16): a half-warp's 8-byte
// gathers are conflict-free. The Hadamard rotation of the activation is done per lane with an
// in-register 64-point FWHT; activations are held as fp16 (scaled by a power of two so they
// cannot overflow) and multiplied with fp16 codebook values by mixed-precision
// fma.rn.f32.f16 into fp32 accumulators.
#include "vq2_common.cuh"

namespace vq2 {

constexpr int DEC_NW = 8;                 // consumer warps
constexpr int DEC_THREADS = (DEC_NW + 1) * 32;
constexpr int DEC_TT = 2;                 // tokens per unit held in registers
constexpr int DEC_STAGES = 4;
constexpr int DEC_GRAN = 8;               // row granule of the work split (keeps copies 16-B sized)
constexpr int CB_COPIES = 16;
constexpr int CB_BYTES = 1024 * 8 * CB_COPIES;   // 128 KB

struct DecodeShared {
  uint64_t full[DEC_STAGES];
  uint64_t empty[DEC_STAGES];
  int nunits;
  int abort;
  short unit_e[VQ2_DECODE_MAX_PAIRS];
  short unit_m[VQ2_DECODE_MAX_PAIRS][DEC_TT];
  int ekey[VQ2_DECODE_MAX_PAIRS];
  int cnt[1024];
};

// ------------------------------------------------------------------ plan: group pairs by expert
// Unit u = (local expert, up to DEC_TT pair indices), units ordered by expert, pairs of an
// expert in pair order. Every CTA builds the same plan.
__device__ void build_plan(const void* ids, int ids_dtype, int M, int E, int expert_base,
                           DecodeShared* sh) {
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int e = tid; e < E; e += nt) sh->cnt[e] = 0;
  for (int u = tid; u < M; u += nt) {
    sh->unit_m[u][0] = -1;
    sh->unit_m[u][1] = -1;
  }
  for (int m = tid; m < M; m += nt) {
    int e = load_id(ids, ids_dtype, m) - expert_base;
    sh->ekey[m] = (e >= 0 && e < E) ? e : -1;
  }
  __syncthreads();
  for (int m = tid; m < M; m += nt) {
    int e = sh->ekey[m];
    if (e >= 0) atomicAdd(&sh->cnt[e], 1);
  }
  __syncthreads();
  if (tid < 32) {  // warp 0: exclusive scan over experts of ceil(cnt/TT) -> unit offsets
    const int per = (E + 31) / 32;
    const int b0 = tid * per;
    int local = 0;
    for (int e = b0; e < min(E, b0 + per); ++e) local += (sh->cnt[e] + DEC_TT - 1) / DEC_TT;
    int incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (tid >= o) incl += v;
    }
    int run = incl - local;
    for (int e = b0; e < min(E, b0 + per); ++e) {
      int c = sh->cnt[e];
      sh->cnt[e] = run;
      run += (c + DEC_TT - 1) / DEC_TT;
    }
    if (tid == 31) sh->nunits = incl;
  }
  __syncthreads();
  for (int m = tid; m < M; m += nt) {
    int e = sh->ekey[m];
    if (e < 0) continue;
    int rank = 0;
    for (int q = 0; q < m; ++q) rank += (sh->ekey[q] == e);
    int u = sh->cnt[e] + rank / DEC_TT;
    sh->unit_e[u] = (short)e;
    sh->unit_m[u][rank % DEC_TT] = (short)m;
  }
  __syncthreads();
}

// ------------------------------------------------------------------ chunk iteration
struct ChunkIter {
  long r, end;       // flattened row position [unit][row]
  int rows_per_unit, S;
  __device__ ChunkIter(long total_rows, int rpu, int S_) : rows_per_unit(rpu), S(S_) {
    long ng = total_rows / DEC_GRAN;
    r = (long)blockIdx.x * ng / gridDim.x * DEC_GRAN;
    end = (long)(blockIdx.x + 1) * ng / gridDim.x * DEC_GRAN;
  }
  __device__ bool next(int& u, int& row0, int& n) {
    if (r >= end) return false;
    u = (int)(r / rows_per_unit);
    row0 = (int)(r % rows_per_unit);
    long lim = min((long)(rows_per_unit - row0), end - r);
    n = (int)min((long)S, lim);
    r += n;
    return true;
  }
};

__device__ __forceinline__ void fill_codebook(const uint16_t* cb, uint8_t* cbs) {
  const uint2* src = (const uint2*)cb;
  for (int idx = threadIdx.x; idx < 1024 * CB_COPIES; idx += blockDim.x) {
    int e = idx / CB_COPIES, c = idx % CB_COPIES;
    *(uint2*)(cbs + e * (8 * CB_COPIES) + c * 8) = src[e];
  }
}

// acc += <codebook[id_s], x_s> over the 16 sub-vectors of one 64-group, for NT tokens.
// lo: the group's 16 index low bytes; hw: its 4 hi bytes; xa[t]: 32 half2 regs of the group.
template <int NT>
__device__ __forceinline__ void group_dot(uint4 lo, uint32_t hw, uint32_t cb_lane,
                                          const uint32_t (*xa)[32], float* acc) {
  const uint32_t lw[4] = {lo.x, lo.y, lo.z, lo.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint32_t L = lw[q];
    const uint32_t hb = hw >> (8 * q);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = 4 * q + j;
      uint32_t off = (((L >> (8 * j)) & 0xFFu) << 7) | (((hb >> (2 * j)) & 3u) << 15);
      uint32_t c0, c1;
      asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(c0), "=r"(c1) : "r"(cb_lane + off));
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        asm("{\n .reg .f16 a0, a1, a2, a3, b0, b1, b2, b3;\n"
            " mov.b32 {a0, a1}, %1;\n mov.b32 {a2, a3}, %2;\n"
            " mov.b32 {b0, b1}, %3;\n mov.b32 {b2, b3}, %4;\n"
            " fma.rn.f32.f16 %0, a0, b0, %0;\n fma.rn.f32.f16 %0, a1, b1, %0;\n"
            " fma.rn.f32.f16 %0, a2, b2, %0;\n fma.rn.f32.f16 %0, a3, b3, %0;\n}"
            : "+f"(acc[t]) : "r"(c0), "r"(c1), "r"(xa[t][2 * s]), "r"(xa[t][2 * s + 1]));
      }
    }
  }
}

// Load one activation row (64*GPL per lane: groups lane + 32 q) as fp32, rotate each group with
// the FWHT, scale into fp16 range and pack. Returns the factor that undoes scale and the 1/8.
template <int GPL, typename LoadF>
__device__ __forceinline__ float load_rotated(LoadF ld, int ngroups, uint32_t (*xa)[32]) {
  const int lane = threadIdx.x & 31;
  float amax = 0.f;
  float v[64];
#pragma unroll
  for (int q = 0; q < GPL; ++q) {
    const int g = lane + 32 * q;
    if (g < ngroups) {
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = ld(g * 64 + i);
      fwht64(v);
#pragma unroll
      for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(v[i]));
    }
  }
  amax = warp_max(amax);
  const float2 sc = f16_range_scale(amax);
#pragma unroll
  for (int q = 0; q < GPL; ++q) {
    const int g = lane + 32 * q;
    if (g < ngroups) {
      // recompute (cheaper in registers than keeping GPL*64 floats live)
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = ld(g * 64 + i);
      fwht64(v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        __half2 h = __floats2half2_rn(v[2 * i] * sc.x, v[2 * i + 1] * sc.x);
        xa[q][i] = *(uint32_t*)&h;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) xa[q][i] = 0u;
    }
  }
  return sc.y * 0.125f;
}

// ------------------------------------------------------------------ kernel A: gate/up + SiLU
template <int GPL>
__global__ void __launch_bounds__(DEC_THREADS, 1)
decode_gateup_kernel(vq2_moe_args a, float* __restrict__ inter) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* cbs = smem;
  DecodeShared* sh = (DecodeShared*)(smem + CB_BYTES);
  uint8_t* stages = smem + CB_BYTES + ((sizeof(DecodeShared) + 127) / 128) * 128;

  pdl_launch_dependents();
  const int H = a.H, I = a.I, M = a.N * a.topk;
  const int nsub = H / 4, ng = H / 64;
  const int S = 8;
  const uint32_t lo_b = S * nsub, hi_b = S * (nsub / 4), sc_b = S * ng * 2;
  const uint32_t stage_b = 2 * (lo_b + hi_b + sc_b);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // zero the output (down kernel accumulates into it after its grid-dependency wait)
  {
    const long tot = (long)a.N * a.H;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < tot; i += (long)gridDim.x * blockDim.x)
      a.out[i] = 0.f;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < DEC_STAGES; ++s) { mbar_init(&sh->full[s], 1); mbar_init(&sh->empty[s], DEC_NW); }
    sh->abort = 0;
    fence_mbar_init();
  }
  fill_codebook(a.w13_cb, cbs);
  build_plan(a.topk_ids, a.ids_dtype, M, a.E, a.expert_base, sh);   // ends with __syncthreads
  const long total = (long)sh->nunits * I;

  if (warp == DEC_NW) {   // ---------------- producer
    if (lane == 0) {
      ChunkIter it(total, I, S);
      int u, i0, n, c = 0;
      while (it.next(u, i0, n)) {
        const int slot = c % DEC_STAGES;
        if (c >= DEC_STAGES && !mbar_wait(&sh->empty[slot], ((c / DEC_STAGES) - 1) & 1)) { sh->abort = 1; break; }
        const long e = sh->unit_e[u];
        const long rg = e * 2 * I + i0, ru = rg + I;
        uint8_t* st = stages + slot * stage_b;
        mbar_arrive_expect_tx(&sh->full[slot], 2u * n * (nsub + nsub / 4 + ng * 2));
        bulk_g2s(st, a.w13_lo + rg * nsub, n * nsub, &sh->full[slot]);
        bulk_g2s(st + lo_b, a.w13_lo + ru * nsub, n * nsub, &sh->full[slot]);
        bulk_g2s(st + 2 * lo_b, a.w13_hi + rg * (nsub / 4), n * (nsub / 4), &sh->full[slot]);
        bulk_g2s(st + 2 * lo_b + hi_b, a.w13_hi + ru * (nsub / 4), n * (nsub / 4), &sh->full[slot]);
        bulk_g2s(st + 2 * (lo_b + hi_b), a.w13_sc + rg * ng, n * ng * 2, &sh->full[slot]);
        bulk_g2s(st + 2 * (lo_b + hi_b) + sc_b, a.w13_sc + ru * ng, n * ng * 2, &sh->full[slot]);
        ++c;
      }
      // drain: every issued copy must land before the CTA exits
      for (int d = max(0, c - DEC_STAGES); d < c; ++d) mbar_wait(&sh->full[d % DEC_STAGES], (d / DEC_STAGES) & 1);
    }
    return;
  }

  // ---------------- consumers
  const uint32_t cb_lane = smem_u32(cbs) + (lane & (CB_COPIES - 1)) * 8;
  uint32_t xa[DEC_TT][GPL][32];
  float inv[DEC_TT];
  int mcur[DEC_TT];
  int ucur = -1;
  ChunkIter it(total, I, S);
  int u, i0, n, c = 0;
  while (it.next(u, i0, n)) {
    const int slot = c % DEC_STAGES;
    if (u != ucur) {
      ucur = u;
#pragma unroll
      for (int t = 0; t < DEC_TT; ++t) {
        const int m = sh->unit_m[u][t];
        mcur[t] = m;
        if (m >= 0) {
          const int tok = m / a.topk;
          const void* xp = a.x;
          const int dt = a.x_dtype;
          inv[t] = load_rotated<GPL>([&](int k) { return load_act(xp, dt, (size_t)tok * H + k); }, ng, xa[t]);
        } else {
          inv[t] = 0.f;
#pragma unroll
          for (int q = 0; q < GPL; ++q)
#pragma unroll
            for (int i = 0; i < 32; ++i) xa[t][q][i] = 0u;
        }
      }
    }
    if (!mbar_wait(&sh->full[slot], (c / DEC_STAGES) & 1)) break;
    const uint8_t* st = stages + slot * stage_b;
    for (int rr = warp; rr < n; rr += DEC_NW) {
      float g[DEC_TT] = {}, up[DEC_TT] = {};
#pragma unroll
      for (int q = 0; q < GPL; ++q) {
        const int gi = lane + 32 * q;
        if (gi < ng) {
          float ag[DEC_TT] = {}, au[DEC_TT] = {};
          const uint4 lg = *(const uint4*)(st + rr * nsub + gi * 16);
          const uint4 lu = *(const uint4*)(st + lo_b + rr * nsub + gi * 16);
          const uint32_t hg = *(const uint32_t*)(st + 2 * lo_b + rr * (nsub / 4) + gi * 4);
          const uint32_t hu = *(const uint32_t*)(st + 2 * lo_b + hi_b + rr * (nsub / 4) + gi * 4);
          const float sg = __half2float(*(const __half*)(st + 2 * (lo_b + hi_b) + (rr * ng + gi) * 2));
          const float su = __half2float(*(const __half*)(st + 2 * (lo_b + hi_b) + sc_b + (rr * ng + gi) * 2));
          uint32_t (*xq)[32] = nullptr;
          (void)xq;
          uint32_t xt[DEC_TT][32];
#pragma unroll
          for (int t = 0; t < DEC_TT; ++t)
#pragma unroll
            for (int i = 0; i < 32; ++i) xt[t][i] = xa[t][q][i];
          group_dot<DEC_TT>(lg, hg, cb_lane, xt, ag);
          group_dot<DEC_TT>(lu, hu, cb_lane, xt, au);
#pragma unroll
          for (int t = 0; t < DEC_TT; ++t) { g[t] += ag[t] * sg; up[t] += au[t] * su; }
        }
      }
#pragma unroll
      for (int t = 0; t < DEC_TT; ++t) {
        const float gs = warp_sum(g[t]) * inv[t];
        const float us = warp_sum(up[t]) * inv[t];
        if (lane == 0 && mcur[t] >= 0)
          inter[(size_t)mcur[t] * I + i0 + rr] = gs / (1.f + __expf(-gs)) * us;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[slot]);
    ++c;
  }
}

// ------------------------------------------------------------------ kernel B: down + combine
template <int GPL>
__global__ void __launch_bounds__(DEC_THREADS, 1)
decode_down_kernel(vq2_moe_args a, const float* __restrict__ inter) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* cbs = smem;
  DecodeShared* sh = (DecodeShared*)(smem + CB_BYTES);
  uint8_t* stages = smem + CB_BYTES + ((sizeof(DecodeShared) + 127) / 128) * 128;

  const int H = a.H, I = a.I, M = a.N * a.topk;
  const int nsub = I / 4, ng = I / 64;
  const int S = 32;
  const uint32_t lo_b = S * nsub, hi_b = S * (nsub / 4), sc_b = S * ng * 2;
  const uint32_t stage_b = lo_b + hi_b + sc_b;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < DEC_STAGES; ++s) { mbar_init(&sh->full[s], 1); mbar_init(&sh->empty[s], DEC_NW); }
    sh->abort = 0;
    fence_mbar_init();
  }
  fill_codebook(a.w2_cb, cbs);
  build_plan(a.topk_ids, a.ids_dtype, M, a.E, a.expert_base, sh);
  const long total = (long)sh->nunits * H;

  if (warp == DEC_NW) {   // ---------------- producer: weights do not depend on the gate/up grid
    if (lane == 0) {
      ChunkIter it(total, H, S);
      int u, h0, n, c = 0;
      while (it.next(u, h0, n)) {
        const int slot = c % DEC_STAGES;
        if (c >= DEC_STAGES && !mbar_wait(&sh->empty[slot], ((c / DEC_STAGES) - 1) & 1)) { sh->abort = 1; break; }
        const long r = (long)sh->unit_e[u] * H + h0;
        uint8_t* st = stages + slot * stage_b;
        mbar_arrive_expect_tx(&sh->full[slot], (uint32_t)n * (nsub + nsub / 4 + ng * 2));
        bulk_g2s(st, a.w2_lo + r * nsub, n * nsub, &sh->full[slot]);
        bulk_g2s(st + lo_b, a.w2_hi + r * (nsub / 4), n * (nsub / 4), &sh->full[slot]);
        bulk_g2s(st + lo_b + hi_b, a.w2_sc + r * ng, n * ng * 2, &sh->full[slot]);
        ++c;
      }
      for (int d = max(0, c - DEC_STAGES); d < c; ++d) mbar_wait(&sh->full[d % DEC_STAGES], (d / DEC_STAGES) & 1);
    }
    return;
  }

  pdl_wait();   // inter and the zeroed output come from the gate/up grid
  const uint32_t cb_lane = smem_u32(cbs) + (lane & (CB_COPIES - 1)) * 8;
  uint32_t xa[DEC_TT][GPL][32];
  float wsc[DEC_TT];
  int tokc[DEC_TT];
  int ucur = -1;
  ChunkIter it(total, H, S);
  int u, h0, n, c = 0;
  while (it.next(u, h0, n)) {
    const int slot = c % DEC_STAGES;
    if (u != ucur) {
      ucur = u;
#pragma unroll
      for (int t = 0; t < DEC_TT; ++t) {
        const int m = sh->unit_m[u][t];
        tokc[t] = m >= 0 ? m / a.topk : -1;
        if (m >= 0) {
          const float* ip = inter + (size_t)m * I;
          wsc[t] = a.topk_w[m] * load_rotated<GPL>([&](int k) { return ip[k]; }, ng, xa[t]);
        } else {
          wsc[t] = 0.f;
#pragma unroll
          for (int q = 0; q < GPL; ++q)
#pragma unroll
            for (int i = 0; i < 32; ++i) xa[t][q][i] = 0u;
        }
      }
    }
    if (!mbar_wait(&sh->full[slot], (c / DEC_STAGES) & 1)) break;
    const uint8_t* st = stages + slot * stage_b;
    for (int rr = warp; rr < n; rr += DEC_NW) {
      float d[DEC_TT] = {};
#pragma unroll
      for (int q = 0; q < GPL; ++q) {
        const int gi = lane + 32 * q;
        if (gi < ng) {
          float ad[DEC_TT] = {};
          const uint4 lo = *(const uint4*)(st + rr * nsub + gi * 16);
          const uint32_t hw = *(const uint32_t*)(st + lo_b + rr * (nsub / 4) + gi * 4);
          const float sc = __half2float(*(const __half*)(st + lo_b + hi_b + (rr * ng + gi) * 2));
          uint32_t xt[DEC_TT][32];
#pragma unroll
          for (int t = 0; t < DEC_TT; ++t)
#pragma unroll
            for (int i = 0; i < 32; ++i) xt[t][i] = xa[t][q][i];
          group_dot<DEC_TT>(lo, hw, cb_lane, xt, ad);
#pragma unroll
          for (int t = 0; t < DEC_TT; ++t) d[t] += ad[t] * sc;
        }
      }
#pragma unroll
      for (int t = 0; t < DEC_TT; ++t) {
        const float ds = warp_sum(d[t]);
        if (lane == 0 && tokc[t] >= 0) atomicAdd(&a.out[(size_t)tokc[t] * H + h0 + rr], ds * wsc[t]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[slot]);
    ++c;
  }
}

static size_t decode_smem_bytes(int S_rows_bytes) {
  return CB_BYTES + ((sizeof(DecodeShared) + 127) / 128) * 128 + (size_t)DEC_STAGES * S_rows_bytes;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace vq2

using namespace vq2;

extern "C" size_t vq2_decode_workspace_size(int N, int topk, int H, int I) {
  (void)H;
  return (size_t)N * topk * I * sizeof(float) + 256;
}

extern "C" int vq2_decode(const vq2_moe_args* a, void* ws, size_t ws_bytes, void* stream) {
  if (!a || !a->x || !a->topk_ids || !a->topk_w || !a->out || !a->w13_cb || !a->w13_lo || !a->w13_hi ||
      !a->w13_sc || !a->w2_cb || !a->w2_lo || !a->w2_hi || !a->w2_sc)
    return VQ2_ERR_NULL;
  if (a->N <= 0 || a->topk <= 0 || a->E <= 0 || a->E > 1024 || a->H % 64 || a->I % 64 || a->H < 64 ||
      a->I < 64 || a->H > 4096 || a->I > 4096)
    return VQ2_ERR_SHAPE;
  if ((long)a->N * a->topk > VQ2_DECODE_MAX_PAIRS) return VQ2_ERR_TOO_MANY_PAIRS;
  if (a->x_dtype < 0 || a->x_dtype > 2 || a->ids_dtype < 0 || a->ids_dtype > 1) return VQ2_ERR_DTYPE;
  const void* ptrs[] = {a->w13_lo, a->w13_hi, a->w13_sc, a->w2_lo, a->w2_hi, a->w2_sc, a->w13_cb, a->w2_cb};
  for (const void* p : ptrs)
    if (!aligned16(p)) return VQ2_ERR_ALIGN;
  if (!ws || ws_bytes < vq2_decode_workspace_size(a->N, a->topk, a->H, a->I)) return VQ2_ERR_WORKSPACE;
  float* inter = (float*)(((uintptr_t)ws + 255) & ~(uintptr_t)255);

  int dev = 0, nsm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return VQ2_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return VQ2_ERR_CUDA;
  cudaStream_t st = (cudaStream_t)stream;

  const int gplA = (a->H / 64 + 31) / 32, gplB = (a->I / 64 + 31) / 32;
  const size_t smA = decode_smem_bytes(8 * 2 * (a->H / 4 + a->H / 16 + a->H / 32));
  const size_t smB = decode_smem_bytes(32 * (a->I / 4 + a->I / 16 + a->I / 32));
  void (*ka)(vq2_moe_args, float*) = gplA == 1 ? decode_gateup_kernel<1> : decode_gateup_kernel<2>;
  void (*kb)(vq2_moe_args, const float*) = gplB == 1 ? decode_down_kernel<1> : decode_down_kernel<2>;
  if (cudaFuncSetAttribute(ka, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smA) != cudaSuccess) return VQ2_ERR_CUDA;
  if (cudaFuncSetAttribute(kb, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smB) != cudaSuccess) return VQ2_ERR_CUDA;

  vq2_moe_args args = *a;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nsm);
  cfg.blockDim = dim3(DEC_THREADS);
  cfg.dynamicSmemBytes = smA;
  cfg.stream = st;
  if (cudaLaunchKernelEx(&cfg, ka, args, inter) != cudaSuccess) return VQ2_ERR_CUDA;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.dynamicSmemBytes = smB;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kb, args, (const float*)inter) != cudaSuccess) return VQ2_ERR_CUDA;
  return VQ2_OK;
}
