// K2 — prefill MoE: grouped GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM)
// (replaces ds4_vq2_cuda.vq2_moe_grouped_wmma, reference vq2_vllm/kernels/ds4_vq2_cuda.py:72-111,
// whose device kernels are vq2_vllm/kernels/vq2_grouped.cu:383-581).
//
// Pipeline of one call (all on the caller's stream, no host sync):
//   align      pairs grouped by expert, each expert padded to 128 slots (csrc/align.cu)
//   act_quant  x -> Hadamard -> per-token quantised activation (fp8 e4m3 with s = 448/amax, as the
//              reference's quant_fp8_rows; or fp16 with a power-of-two range scale)
//   gateup     per (128-slot block, 128 gate + 128 matching up rows): D = A . B^T in TMEM, epilogue
//              inter = silu(g * inv_x) * (u * inv_x)   (reference vq2_grouped.cu:255-264 fused)
//   vb_quant   inter -> Hadamard -> per-slot quantised activation (+ inv)
//   down       per (block, 256 output rows): D = vb . Wd^T; epilogue out[tok] += D * w * inv_vb
//
// GEMM CTA (608 threads; one 128-token block pair and one 256-row weight tile): warp 0 loads the
// activation tiles of the pass's blocks (rows in slot order, 128-byte swizzled K-major) with 2-D
// TMA into a 2-stage ring; warp 1 loads the weight tile's index planes (the lo plane by 2-D TMA,
// the small hi / scale planes with cp.async signalling the same mbarrier) into a 3-stage ring;
// warp 2 lane 0 issues tcgen05.mma (M=128 tokens, N=256 = 128 gate + 128 up rows or 256 down rows,
// K=32 fp8 / K=16 f16 per instruction) into fp32 TMEM accumulators, one per block (512 columns
// for two blocks of the same expert, so every decoded weight tile feeds two MMAs); warps 3..18
// decode the weight tile (10-bit index -> fp16 codebook vector x fp16 group scale -> e4m3 / f16)
// straight into the swizzled B tile of a 2-stage ring and then run the epilogue out of TMEM.
// tcgen05.commit frees the ring stages; the codebook (8 copies, lane l reads copy l mod 8)
// arrives by one bulk copy and is replicated in shared memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp8.h>
#include <algorithm>
#include "vq2_common.cuh"

namespace vq2 {

int launch_align_ex(const void* ids, int dt, long N, int k, int E, int BM, int base, int drop, int32_t* st,
                    int32_t* ss, uint8_t* val, int32_t* be, int* counts, cudaStream_t stream, int2* ranges);

// ------------------------------------------------------------------ tcgen05 helpers
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms 1024 B apart (stride
// byte offset), leading byte offset unused for this layout (1), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                 "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                 "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                 "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile("cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool ok) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ------------------------------------------------------------------ weight decode into registers
// Exact fp32 products of two f16 values (sm_100 mixed-precision FMA; the product of two 11-bit
// significands fits fp32, and the -0 addend keeps the sign of a zero product): (h2.lo * s, h2.hi * s).
__device__ __forceinline__ float2 f16x2_times_f16(uint32_t h2, unsigned short s) {
  float2 r;
  asm("{\n .reg .b16 a, b;\n mov.b32 {a, b}, %2;\n fma.rn.f32.f16 %0, a, %3, %4;\n fma.rn.f32.f16 %1, b, %3, %4;\n}"
      : "=f"(r.x), "=f"(r.y) : "r"(h2), "h"(s), "f"(-0.0f));
  return r;
}

// fp8: 8 sub-vectors of a weight row (lo: their 8 low index bytes, hw: their 2 hi bytes in the
// low 16 bits, sb: the f16 bits of the group scale) -> 8 words of 4 e4m3 values,
// e4m3(sat(C[id] * sc)) with the product exact in fp32 and one rounding (reference
// vq2_grouped.cu:434-446). cbl: this lane's codebook copy (entries 128 bytes apart: 16 copies,
// lane l reads copy l mod 16, so a warp's 8-byte gathers are conflict-free).
__device__ __forceinline__ void decode8_fp8(uint32_t cbl, uint2 lo, uint32_t hw, unsigned short sb, uint32_t* v) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint32_t ids[2];
    unpack_ids4(q ? lo.y : lo.x, (hw >> (8 * q)) & 0xFFu, ids[0], ids[1]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t id = (j & 2) ? (ids[j & 1] >> 16) : (ids[j & 1] & 0xFFFFu);
      const uint2 c = lds64(cbl + (id << 7));
      const __nv_fp8x2_storage_t p0 = __nv_cvt_float2_to_fp8x2(f16x2_times_f16(c.x, sb), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t p1 = __nv_cvt_float2_to_fp8x2(f16x2_times_f16(c.y, sb), __NV_SATFINITE, __NV_E4M3);
      v[4 * q + j] = (uint32_t)p0 | ((uint32_t)p1 << 16);
    }
  }
}

// fp8: the 16 sub-vectors of one 64-group (one scale) -> 16 words.
__device__ __forceinline__ void decode16_fp8(uint32_t cbl, uint4 lo, uint32_t hw, unsigned short sb, uint32_t* v) {
  decode8_fp8(cbl, make_uint2(lo.x, lo.y), hw & 0xFFFFu, sb, v);
  decode8_fp8(cbl, make_uint2(lo.z, lo.w), hw >> 16, sb, v + 8);
}

// f16: 4 sub-vectors of a row (lo: 4 low index bytes, hw: 1 hi byte) -> 8 words of 2 f16 values,
// C[id] * sc in fp16.
__device__ __forceinline__ void decode4_f16(uint32_t cbl, uint32_t lo, uint32_t hw, unsigned short sb, uint32_t* v) {
  const __half2 s2 = __half2half2(__ushort_as_half(sb));
  uint32_t ids[2];
  unpack_ids4(lo, hw & 0xFFu, ids[0], ids[1]);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t id = (j & 2) ? (ids[j & 1] >> 16) : (ids[j & 1] & 0xFFFFu);
    const uint2 c = lds64(cbl + (id << 7));
    const __half2 a0 = __hmul2(*(const __half2*)&c.x, s2), a1 = __hmul2(*(const __half2*)&c.y, s2);
    v[2 * j] = *(const uint32_t*)&a0;
    v[2 * j + 1] = *(const uint32_t*)&a1;
  }
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
               ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
               ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
                 "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
               : "memory");
}
__device__ __forceinline__ void keep_live16(const uint32_t* v) {
  asm volatile("" ::"r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
               "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]));
}
// An empty statement that reads 8 registers: keeps them allocated (unmodified) up to this point.
__device__ __forceinline__ void keep_live8(const uint32_t* v) {
  asm volatile("" ::"r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]));
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (TMEM) += A (TMEM, M = 128 weight rows, K-major) . B (shared memory descriptor, N slots)^T
template <int PREC>
__device__ __forceinline__ void umma_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc,
                                            uint32_t acc) {
  if (PREC == VQ2_PREC_FP8)
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n}"
                 ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
  else
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}"
                 ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}

// ------------------------------------------------------------------ grouped GEMM kernel
// Persistent; one CTA per SM walks the work list w = blockIdx.x, blockIdx.x + gridDim.x, ...
// (w -> chunk w / T, row tile w % T; chunks heaviest first). A work item is one chunk of up to
// P2_NMAX consecutive slots of one expert (its tokens, padded to P2_BM) against P2_NT x 128
// weight rows: GATEUP = 128 gate rows and the 128 matching up rows of tile t; otherwise 256
// down rows. Per 128-byte K stage the decoder warps write the decoded rows into tensor memory
// (the MMA's A operand, one 128-lane tile per 128 rows), warp 0 loads the chunk's activation rows
// by TMA (B operand), warp 2 issues M=128 x N=slots MMAs into one TMEM accumulator per row tile.
// The epilogue reads the accumulators (lane = weight row, column = slot): gate/up writes
// inter[slot][i] = silu(g * inv) * (u * inv) (reference vq2_grouped.cu:255-264); down adds
// acc * w * inv_vb into out[token] with fp32 reductions.
constexpr int P2_ROWS = 128;                 // weight rows per A tile (MMA M)
constexpr int P2_NT = 2;                     // A tiles per work item
constexpr int P2_NMAX = 192;                 // slots per chunk (MMA N at most)
constexpr int P2_BM = 32;                    // per-expert slot padding (moe_align block)
constexpr int P2_CHUNK_BLOCKS = P2_NMAX / P2_BM;
constexpr int P2_BSTAGES = 2, P2_ISTAGES = 3, P2_ASTAGES = 2;
constexpr int P2_DEC_WARPS = 16;            // 4 per TMEM lane quarter: row tile x K half
constexpr int P2_THREADS = (3 + P2_DEC_WARPS) * 32;
constexpr int P2_BTILE = P2_NMAX * 128;      // one B stage: 192 slot rows x 128 bytes (SW128)
constexpr int P2_CB_COPIES = 16;
constexpr int P2_CB_BYTES = 1024 * 8 * P2_CB_COPIES;
constexpr int P2_IDX = 11264;                // index planes of one stage: lo 256 x 32, hi 256 x 8, sc 256 x 4
constexpr int P2_IDX_HI = 8192, P2_IDX_SC = 10240;
constexpr uint32_t P2_TMEM_COLS = 512;
// TMEM columns: accumulator of tile 0 at 0 (N <= 192), A stage 0 at 192 (2 tiles x 32 columns),
// accumulator of tile 1 at 256, A stage 1 at 448.
__host__ __device__ constexpr uint32_t p2_acc_col(int t) { return t ? 256u : 0u; }
__host__ __device__ constexpr uint32_t p2_a_col(int s, int t) { return (s ? 448u : 192u) + 32u * t; }

struct P2Shared {
  uint64_t full_b[P2_BSTAGES], empty_b[P2_BSTAGES];
  uint64_t full_i[P2_ISTAGES], empty_i[P2_ISTAGES];
  uint64_t full_a[P2_ASTAGES], empty_a[P2_ASTAGES];
  uint64_t done, acc_empty, cbbar, drain;
  uint32_t tmem_base;
  int abort;
};
constexpr size_t P2_SMEM = (size_t)P2_CB_BYTES + (size_t)P2_BSTAGES * P2_BTILE + (size_t)P2_ISTAGES * P2_IDX +
                           sizeof(P2Shared) + 1024;
static_assert(P2_SMEM <= 227 * 1024, "prefill GEMM shared memory");

struct P2Args {
  const int4* chunks;        // {expert, first slot, slots, 0}, heaviest first
  const int* nchunks;        // device count of chunks
  const float* inv_slot;     // per slot: inverse quantisation scale of its activation row
  const int32_t* st;         // sorted_tok [Pmax]
  const int32_t* ss;         // sorted_slot [Pmax]
  const uint8_t* val;        // valid [Pmax]
  const uint8_t* lo;
  const uint8_t* hi;
  const uint16_t* sc;
  const uint16_t* cb;
  const float* topk_w;
  float* inter;              // gate/up output [Pmax, I]
  float* out;                // down output [N, H]
  int K;                     // input width (elements)
  int R;                     // weight rows per expert (2I or H)
  int I, H, topk;
  int T;                     // row tiles per chunk
};

// weight row of A tile t, lane r, for row tile `tile` of expert e
template <bool GATEUP>
__device__ __forceinline__ long p2_weight_row(const P2Args& a, int e, int tile, int t, int r) {
  if (GATEUP) return (long)e * a.R + (long)t * a.I + tile * P2_ROWS + r;
  return (long)e * a.R + (long)tile * (P2_NT * P2_ROWS) + t * P2_ROWS + r;
}

template <int PREC, bool GATEUP>
__global__ void __launch_bounds__(P2_THREADS, 1)
prefill_gemm_kernel(P2Args a, const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_lo) {
  extern __shared__ __align__(1024) uint8_t p2_smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)p2_smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* cbs = smem;
  uint8_t* btiles = smem + P2_CB_BYTES;
  uint8_t* itiles = btiles + P2_BSTAGES * P2_BTILE;
  P2Shared* sh = (P2Shared*)(itiles + P2_ISTAGES * P2_IDX);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int elem = PREC == VQ2_PREC_FP8 ? 1 : 2;
  constexpr int KE = 128 / elem;               // K elements per stage (128 bytes)
  constexpr int LOB = KE / 4;                  // lo bytes per row per stage
  const int nstage = a.K / KE;
  const int nsub = a.K / 4, ngk = a.K / 64;
  const int nwork = *a.nchunks * a.T;
  auto B_t = [&](int slot) { return btiles + slot * P2_BTILE; };
  auto I_t = [&](int slot) { return itiles + slot * P2_IDX; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < P2_BSTAGES; ++s) { mbar_init(&sh->full_b[s], 1); mbar_init(&sh->empty_b[s], 1); }
    for (int s = 0; s < P2_ISTAGES; ++s) { mbar_init(&sh->full_i[s], 33); mbar_init(&sh->empty_i[s], P2_DEC_WARPS); }
    for (int s = 0; s < P2_ASTAGES; ++s) { mbar_init(&sh->full_a[s], P2_DEC_WARPS); mbar_init(&sh->empty_a[s], 1); }
    mbar_init(&sh->done, 1);
    mbar_init(&sh->acc_empty, P2_DEC_WARPS);
    mbar_init(&sh->cbbar, 1);
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(&sh->cbbar, 1024 * 8);
    bulk_g2s(B_t(0), a.cb, 1024 * 8, &sh->cbbar);     // the codebook lands in a B stage first
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&sh->tmem_base)), "r"(P2_TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  if (!mbar_wait(&sh->cbbar, 0)) sh->abort = 1;
  {  // replicate: entry e of copy c at e * 128 + c * 8; consecutive 16-byte stores
    const uint2* src = (const uint2*)B_t(0);
    for (int idx = threadIdx.x; idx < 1024 * (P2_CB_COPIES / 2); idx += blockDim.x) {
      const uint2 v = src[idx / (P2_CB_COPIES / 2)];
      *(uint4*)(cbs + idx * 16) = make_uint4(v.x, v.y, v.x, v.y);
    }
  }
  tc_fence_before();
  __syncthreads();                                     // codebook ready, B stage 0 free again
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  volatile int* abort = &sh->abort;

  if (warp == 0) {
    // ---------------- activation loader (lane 0): B stages of each item by TMA
    if (lane == 0) {
      int gb = 0;
      for (int w = blockIdx.x; w < nwork && !*abort; w += gridDim.x) {
        const int4 ch = a.chunks[w / a.T];
        for (int c = 0; c < nstage; ++c, ++gb) {
          const int slot = gb % P2_BSTAGES;
          if (gb >= P2_BSTAGES && !mbar_wait(&sh->empty_b[slot], ((gb / P2_BSTAGES) - 1) & 1)) { *abort = 1; break; }
          mbar_arrive_expect_tx(&sh->full_b[slot], P2_BTILE);
          tma_load_2d(B_t(slot), &tm_act, c * 128, ch.y, &sh->full_b[slot]);
        }
      }
      // every issued load has landed before the CTA can exit
      for (int q = max(0, gb - P2_BSTAGES); q < gb; ++q) mbar_wait(&sh->full_b[q % P2_BSTAGES], (q / P2_BSTAGES) & 1);
    }
  } else if (warp == 1) {
    // ---------------- index loader: lo plane by TMA (two 128-row boxes), hi / scale planes by cp.async
    int gi = 0;
    for (int w = blockIdx.x; w < nwork && !*abort; w += gridDim.x) {
      const int e = a.chunks[w / a.T].x, tile = w % a.T;
      // this lane's rows are lane + 32 i (i < 4: tile 0, else tile 1); hi / scale row pointers
      // are formed from one base per tile
      const long wr0 = p2_weight_row<GATEUP>(a, e, tile, 0, lane), wr1 = p2_weight_row<GATEUP>(a, e, tile, 1, lane);
      const uint8_t* hi_b0 = a.hi + wr0 * (nsub / 4);
      const uint8_t* hi_b1 = a.hi + wr1 * (nsub / 4);
      const uint8_t* sc_b0 = (const uint8_t*)(a.sc + wr0 * ngk);
      const uint8_t* sc_b1 = (const uint8_t*)(a.sc + wr1 * ngk);
      const long hi_step = 32L * (nsub / 4), sc_step = 32L * ngk * 2;
      const int row0 = (int)p2_weight_row<GATEUP>(a, e, tile, 0, 0);
      const int row1 = (int)p2_weight_row<GATEUP>(a, e, tile, 1, 0);
      for (int c = 0; c < nstage; ++c, ++gi) {
        const int slot = gi % P2_ISTAGES;
        if (gi >= P2_ISTAGES && !mbar_wait(&sh->empty_i[slot], ((gi / P2_ISTAGES) - 1) & 1)) { *abort = 1; break; }
        const uint32_t ibase = smem_u32(I_t(slot));
        if (lane == 0) {
          mbar_arrive_expect_tx(&sh->full_i[slot], P2_NT * P2_ROWS * LOB);
          tma_load_2d(I_t(slot), &tm_lo, c * LOB, row0, &sh->full_i[slot]);
          tma_load_2d(I_t(slot) + P2_ROWS * LOB, &tm_lo, c * LOB, row1, &sh->full_i[slot]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int R = lane + 32 * i;
          const uint8_t* hi_r = (i < 4 ? hi_b0 : hi_b1) + (i & 3) * hi_step;
          const uint8_t* sc_r = (i < 4 ? sc_b0 : sc_b1) + (i & 3) * sc_step;
          if (PREC == VQ2_PREC_FP8) {          // hi: 8 bytes (32 sub-vectors); scales of 2 groups
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(ibase + P2_IDX_HI + R * 8), "l"(hi_r + c * 8) : "memory");
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + P2_IDX_SC + R * 4), "l"(sc_r + c * 4) : "memory");
          } else {                             // hi: 4 bytes (16 sub-vectors); the scale pair holding this group
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + P2_IDX_HI + R * 8), "l"(hi_r + c * 4) : "memory");
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + P2_IDX_SC + R * 4), "l"(sc_r + (c & ~1) * 2) : "memory");
          }
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&sh->full_i[slot])) : "memory");
      }
    }
    cp_async_wait<0>();
    if (lane == 0)   // the lo-plane TMA loads of the last stages have landed
      for (int q = max(0, gi - P2_ISTAGES); q < gi; ++q) mbar_wait(&sh->full_i[q % P2_ISTAGES], (q / P2_ISTAGES) & 1);
  } else if (warp == 2) {
    // ---------------- MMA issuer (lane 0)
    if (lane == 0) {
      int gb = 0, ga = 0, it = 0;
      for (int w = blockIdx.x; w < nwork && !*abort; w += gridDim.x, ++it) {
        const int ns = a.chunks[w / a.T].z;
        const uint32_t idesc = (1u << 4) | ((uint32_t)(ns >> 3) << 17) | ((uint32_t)(P2_ROWS >> 4) << 24);
        if (it > 0 && !mbar_wait(&sh->acc_empty, (it - 1) & 1)) { *abort = 1; break; }
        tc_fence_after();
        bool ok = true;
        for (int c = 0; c < nstage; ++c, ++gb, ++ga) {
          const int bslot = gb % P2_BSTAGES, aslot = ga % P2_ASTAGES;
          if (!mbar_wait(&sh->full_b[bslot], (gb / P2_BSTAGES) & 1) ||
              !mbar_wait(&sh->full_a[aslot], (ga / P2_ASTAGES) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t bbase = smem_u32(B_t(bslot));
#pragma unroll
          for (int t = 0; t < P2_NT; ++t)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_tmem_a<PREC>(tmem + p2_acc_col(t), tmem + p2_a_col(aslot, t) + 8 * ks,
                                umma_desc_sw128(bbase + ks * 32), idesc, (c | ks) != 0);
          umma_commit(&sh->empty_b[bslot]);
          umma_commit(&sh->empty_a[aslot]);
        }
        umma_commit(&sh->done);       // arrives once every MMA issued so far has completed
        if (!ok) { *abort = 1; break; }
      }
      umma_commit(&sh->drain);        // nothing of ours still reads TMEM or shared memory after this
      mbar_wait(&sh->drain, 0);
    }
  } else {
    // ---------------- decoders (16 warps): warp -> TMEM lane quarter q, row tile t, K half h
    // Software-pipelined by one stage: the tensor-memory store of stage c is issued, then stage
    // c + 1's index planes are read and decoded into registers, and only then is the store of
    // stage c waited for and the stage handed to the MMA warp, so the store latency does not sit
    // on the decode chain.
    const int q = warp & 3, j = (warp - 3) >> 2, t = j >> 1, h = j & 1;
    const int r = q * 32 + lane, R = t * P2_ROWS + r;
    const uint32_t cbl = smem_u32(cbs) + (lane & (P2_CB_COPIES - 1)) * 8;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    int gi = 0, ga = 0, it = 0;
    // stage gi of the index ring -> 16 decoded words (this thread's row, K half), then frees the
    // slot (after the decode consumed every lane's loads of it: the next writer is the loader's
    // TMA / cp.async)
    auto decode_stage = [&](int c, uint32_t* v) -> bool {
      const int islot = gi % P2_ISTAGES;
      if (!mbar_wait(&sh->full_i[islot], (gi / P2_ISTAGES) & 1)) return false;
      const uint32_t ip = smem_u32(I_t(islot));
      if (PREC == VQ2_PREC_FP8) {             // one 64-group: 16 sub-vectors
        const uint4 lo = lds128_v(ip + R * 32 + h * 16);
        const uint32_t hw = lds32_v(ip + P2_IDX_HI + R * 8 + h * 4);
        const uint32_t sbits = lds16_v(ip + P2_IDX_SC + R * 4 + h * 2);
        decode16_fp8(cbl, lo, hw, (unsigned short)sbits, v);
      } else {                                // half of a 64-group: 8 sub-vectors
        const uint2 lo = lds64_v(ip + R * 16 + h * 8);
        const uint32_t hw = lds16_v(ip + P2_IDX_HI + R * 8 + h * 2);
        const uint32_t sbits = lds16_v(ip + P2_IDX_SC + R * 4 + (c & 1) * 2);
        decode4_f16(cbl, lo.x, hw, (unsigned short)sbits, v);
        decode4_f16(cbl, lo.y, hw >> 8, (unsigned short)sbits, v + 8);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty_i[islot]);
      ++gi;
      return true;
    };
    for (int w = blockIdx.x; w < nwork; w += gridDim.x, ++it) {
      const int4 ch = a.chunks[w / a.T];
      const int tile = w % a.T;
      bool ok = !*abort;
      // two register sets: a tcgen05.st reads its source registers asynchronously, so the set
      // being stored stays untouched (and is kept live) until its tcgen05.wait::st
      uint32_t va[16], vb[16];
      if (ok) ok = decode_stage(0, va);
      auto step = [&](int c, uint32_t* cur, uint32_t* nxt) {
        const int aslot = ga % P2_ASTAGES;
        if (ga >= P2_ASTAGES && !mbar_wait(&sh->empty_a[aslot], ((ga / P2_ASTAGES) - 1) & 1)) { ok = false; return; }
        tc_fence_after();
        tmem_st16(tmem + tlane + p2_a_col(aslot, t) + 16 * h, cur);
        if (c + 1 < nstage && !decode_stage(c + 1, nxt)) ok = false;
        tmem_st_wait();
        keep_live16(cur);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sh->full_a[aslot]);
        ++ga;
      };
      for (int c = 0; c < nstage && ok; c += 2) {
        step(c, va, vb);
        if (c + 1 < nstage && ok) step(c + 1, vb, va);
      }
      if (!ok) *abort = 1;
      if (*abort) break;
      // ---------------- epilogue of the item out of TMEM (lane = weight row, column = slot)
      if (!mbar_wait(&sh->done, it & 1)) { *abort = 1; break; }
      tc_fence_after();
      const int ncol = ch.z >> 5;                          // 32-slot column groups
      if (GATEUP) {
        for (int cg = j; cg < ncol; cg += 4) {
          const int s0 = ch.y + cg * 32;
          const float myinv = a.inv_slot[s0 + lane];
          float* dst = a.inter + (size_t)s0 * a.I + tile * P2_ROWS + r;
#pragma unroll 1
          for (int hh = 0; hh < 4; ++hh) {          // 8 columns at a time (register budget)
            float g[8], u[8];
            tmem_ld8(tmem + tlane + p2_acc_col(0) + cg * 32 + hh * 8, g);
            tmem_ld8(tmem + tlane + p2_acc_col(1) + cg * 32 + hh * 8, u);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float inv = __shfl_sync(0xffffffffu, myinv, hh * 8 + k);
              const float gg = g[k] * inv, uu = u[k] * inv;
              dst[(size_t)(hh * 8 + k) * a.I] = __fdividef(gg, 1.f + __expf(-gg)) * uu;
            }
          }
        }
      } else {
        for (int u = j; u < P2_NT * ncol; u += 4) {
          const int tt = u & 1, cg = u >> 1;
          const int s = ch.y + cg * 32 + lane;
          const int mytok = a.val[s] ? a.st[s] : -1;
          const float myw = mytok >= 0 ? a.topk_w[(size_t)mytok * a.topk + a.ss[s]] * a.inv_slot[s] : 0.f;
          float* col = a.out + tile * (P2_NT * P2_ROWS) + tt * P2_ROWS + r;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {          // 16 columns at a time (register budget)
            float v[16];
            tmem_ld16(tmem + tlane + p2_acc_col(tt) + cg * 32 + hh * 16, v);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int tok = __shfl_sync(0xffffffffu, mytok, hh * 16 + k);
              const float wk = __shfl_sync(0xffffffffu, myw, hh * 16 + k);
              if (tok >= 0) atomicAdd(col + (size_t)tok * a.H, v[k] * wk);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->acc_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P2_TMEM_COLS) : "memory");
  }
}

// ------------------------------------------------------------------ work list
// One CTA, a thread per expert: the chunks of every expert's padded slot range (from moe_align),
// at most P2_NMAX slots each, ordered by size, largest first.
__global__ void __launch_bounds__(1024) build_chunks_kernel(const int2* __restrict__ ranges, int E,
                                                            int4* __restrict__ chunks, int* __restrict__ nchunks) {
  __shared__ int cnt[P2_CHUNK_BLOCKS + 1], base[P2_CHUNK_BLOCKS + 1];
  if (threadIdx.x <= P2_CHUNK_BLOCKS) cnt[threadIdx.x] = 0;
  __syncthreads();
  for (int pass = 0; pass < 2; ++pass) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const int2 rg = ranges[e];
      for (int k = 0; k < rg.y; k += P2_NMAX) {
        const int size = min(P2_NMAX, rg.y - k) / P2_BM;
        if (pass == 0) {
          atomicAdd(&cnt[size], 1);
        } else {
          const int pos = base[size] + atomicAdd(&cnt[size], 1);
          chunks[pos] = make_int4(e, rg.x + k, size * P2_BM, 0);
        }
      }
    }
    __syncthreads();
    if (pass == 0 && threadIdx.x == 0) {
      int run = 0;
      for (int size = P2_CHUNK_BLOCKS; size >= 1; --size) { base[size] = run; run += cnt[size]; cnt[size] = 0; }
      *nchunks = run;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ activation quantisation
// One CTA (8 warps) per row: y = x @ H per 64-group (shuffle FWHT, lane holds elements lane and
// lane + 32 of each group), then fp8: s = 448 / max(amax, 1e-6), q = e4m3(y * s), inv = 1 / s
// (reference quant_fp8_rows, ds4_vq2_cuda.py:11-23, applied to had_act_batch output as at
// ds4_vq2_cuda.py:94 and :106); f16: s = the power of two with amax * s <= 2^15, q = f16(y * s).
// Rows with valid[row] == 0 are written as zeros with inv = 0. cols <= 4096.
template <int PREC>
__global__ void __launch_bounds__(256) had_quant_rows_kernel(const void* __restrict__ x, int in_dt,
                                                             const uint8_t* __restrict__ valid, int cols,
                                                             uint8_t* __restrict__ out, float* __restrict__ inv) {
  __shared__ float red[33];
  const long row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ng = cols / 64;
  const int elem = PREC == VQ2_PREC_FP8 ? 1 : 2;
  uint8_t* orow = out + row * (size_t)cols * elem;
  if (valid && !valid[row]) {
    for (int c = threadIdx.x; c < cols * elem / 4; c += blockDim.x) ((uint32_t*)orow)[c] = 0u;
    if (threadIdx.x == 0) inv[row] = 0.f;
    return;
  }
  float va[8], vb[8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int g = warp + 8 * i;
    va[i] = vb[i] = 0.f;
    if (g < ng) {
      const size_t base = row * (size_t)cols + g * 64;
      float a = load_act(x, in_dt, base + lane), b = load_act(x, in_dt, base + 32 + lane);
      float t = a + b;
      b = a - b;
      a = t;
#pragma unroll
      for (int len = 16; len >= 1; len >>= 1) {
        const float pa = __shfl_xor_sync(0xffffffffu, a, len), pb = __shfl_xor_sync(0xffffffffu, b, len);
        a = (lane & len) ? (pa - a) : (a + pa);
        b = (lane & len) ? (pb - b) : (b + pb);
      }
      va[i] = a * 0.125f;
      vb[i] = b * 0.125f;
      amax = fmaxf(amax, fmaxf(fabsf(va[i]), fabsf(vb[i])));
    }
  }
  amax = block_max(amax, red);
  float s;
  if (PREC == VQ2_PREC_FP8) {
    s = 448.0f / fmaxf(amax, 1e-6f);
  } else {
    s = 1.f;
    if (amax > 0.f) {
      int ex;
      frexpf(32768.f / amax, &ex);
      s = ldexpf(1.f, max(-100, min(100, ex - 1)));
    }
  }
  if (threadIdx.x == 0) inv[row] = 1.0f / s;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int g = warp + 8 * i;
    if (g < ng) {
      if (PREC == VQ2_PREC_FP8) {
        orow[g * 64 + lane] = (uint8_t)__nv_cvt_float_to_fp8(va[i] * s, __NV_SATFINITE, __NV_E4M3);
        orow[g * 64 + 32 + lane] = (uint8_t)__nv_cvt_float_to_fp8(vb[i] * s, __NV_SATFINITE, __NV_E4M3);
      } else {
        ((__half*)orow)[g * 64 + lane] = __float2half_rn(va[i] * s);
        ((__half*)orow)[g * 64 + 32 + lane] = __float2half_rn(vb[i] * s);
      }
    }
  }
}

// Quantised token rows into slot order (padding slots zero) with their inverse scales, so the
// activation rows of a chunk are one contiguous 2-D TMA box.
__global__ void __launch_bounds__(256) gather_slot_rows_kernel(const uint8_t* __restrict__ src,
                                                              const float* __restrict__ inv_tok,
                                                              const int32_t* __restrict__ st,
                                                              const uint8_t* __restrict__ val, int row_bytes,
                                                              uint8_t* __restrict__ dst, float* __restrict__ inv_slot) {
  const long p = blockIdx.x;
  uint4* d = (uint4*)(dst + p * (size_t)row_bytes);
  const bool ok = val[p] != 0;
  const int tok = ok ? st[p] : 0;
  const uint4* s = (const uint4*)(src + (size_t)tok * row_bytes);
  for (int i = threadIdx.x; i < row_bytes / 16; i += blockDim.x) d[i] = ok ? s[i] : make_uint4(0, 0, 0, 0);
  if (threadIdx.x == 0) inv_slot[p] = ok ? inv_tok[tok] : 0.f;
}

// ------------------------------------------------------------------ host
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int encode_2d(CUtensorMap* m, const void* base, uint64_t inner_bytes, uint64_t rows, uint32_t box_x,
                     uint32_t box_y, bool swizzle128) {
  if (!g_encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return VQ2_ERR_CUDA;
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  }
  const cuuint64_t dims[2] = {inner_bytes, rows};
  const cuuint64_t strides[1] = {inner_bytes};
  const cuuint32_t box[2] = {box_x, box_y};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? VQ2_OK : VQ2_ERR_CUDA;
}

struct PfLayout {
  long M, Pmax, nblk, nchunks_align;
  size_t off_st, off_ss, off_val, off_be, off_counts, off_xq, off_invx, off_xs, off_invxs, off_inter, off_vb,
      off_invvb, off_chunks, off_nchunks, off_ranges, total;
};

static size_t up256(size_t v) { return (v + 255) & ~(size_t)255; }

static PfLayout pf_layout(int N, int k, int E, int H, int I, int prec) {
  PfLayout L;
  const size_t elem = prec == VQ2_PREC_FP8 ? 1 : 2;
  L.M = (long)N * k;
  L.Pmax = L.M + (long)std::min<long>(L.M, E) * P2_BM;
  L.nblk = L.Pmax / P2_BM;
  L.nchunks_align = std::max<long>(1, (L.M + 8191) / 8192);
  size_t o = 0;
  L.off_st = o; o = up256(o + L.Pmax * 4);
  L.off_ss = o; o = up256(o + L.Pmax * 4);
  L.off_val = o; o = up256(o + L.Pmax);
  L.off_be = o; o = up256(o + L.nblk * 4);
  L.off_counts = o; o = up256(o + L.nchunks_align * E * 4);
  L.off_xq = o; o = up256(o + (size_t)N * H * elem);
  L.off_invx = o; o = up256(o + (size_t)N * 4);
  L.off_xs = o; o = up256(o + (size_t)L.Pmax * H * elem);
  L.off_invxs = o; o = up256(o + (size_t)L.Pmax * 4);
  L.off_inter = o; o = up256(o + (size_t)L.Pmax * I * 4);
  L.off_vb = o; o = up256(o + (size_t)L.Pmax * I * elem);
  L.off_invvb = o; o = up256(o + (size_t)L.Pmax * 4);
  L.off_chunks = o; o = up256(o + (size_t)L.nblk * 16);
  L.off_nchunks = o; o = up256(o + 4);
  L.off_ranges = o; o = up256(o + (size_t)E * 8);
  L.total = o + 256;
  return L;
}

static bool g_pf_attr[64];

}  // namespace vq2

using namespace vq2;

extern "C" size_t vq2_prefill_workspace_size(int N, int topk, int E, int H, int I, int precision) {
  if (N <= 0 || topk <= 0 || E <= 0) return 0;
  return pf_layout(N, topk, E, H, I, precision).total;
}

extern "C" int vq2_prefill(const vq2_moe_args* a, int prec, void* ws, size_t ws_bytes, void* stream) {
  if (!a || !a->x || !a->topk_ids || !a->topk_w || !a->out || !a->w13_cb || !a->w13_lo || !a->w13_hi ||
      !a->w13_sc || !a->w2_cb || !a->w2_lo || !a->w2_hi || !a->w2_sc)
    return VQ2_ERR_NULL;
  if (prec != VQ2_PREC_FP8 && prec != VQ2_PREC_F16) return VQ2_ERR_DTYPE;
  if (a->N <= 0 || a->topk <= 0 || a->E <= 0 || a->E > 1024 || a->H % 256 || a->I % 128 || a->H > 4096 ||
      a->I > 4096)
    return VQ2_ERR_SHAPE;
  if (a->x_dtype < 0 || a->x_dtype > 2 || a->ids_dtype < 0 || a->ids_dtype > 1) return VQ2_ERR_DTYPE;
  const void* ptrs[] = {a->w13_lo, a->w13_hi, a->w13_sc, a->w2_lo, a->w2_hi, a->w2_sc, a->w13_cb, a->w2_cb};
  for (const void* p : ptrs)
    if (((uintptr_t)p & 15) != 0) return VQ2_ERR_ALIGN;
  const PfLayout L = pf_layout(a->N, a->topk, a->E, a->H, a->I, prec);
  if (L.Pmax > (1L << 30)) return VQ2_ERR_SHAPE;
  if (!ws || ws_bytes < L.total) return VQ2_ERR_WORKSPACE;
  uint8_t* w = (uint8_t*)(((uintptr_t)ws + 255) & ~(uintptr_t)255);
  int32_t* st = (int32_t*)(w + L.off_st);
  int32_t* ss = (int32_t*)(w + L.off_ss);
  uint8_t* val = w + L.off_val;
  int32_t* be = (int32_t*)(w + L.off_be);
  int* counts = (int*)(w + L.off_counts);
  uint8_t* xq = w + L.off_xq;
  uint8_t* xs = w + L.off_xs;
  float* invx = (float*)(w + L.off_invx);
  float* invxs = (float*)(w + L.off_invxs);
  float* inter = (float*)(w + L.off_inter);
  uint8_t* vb = w + L.off_vb;
  float* invvb = (float*)(w + L.off_invvb);
  int4* chunks = (int4*)(w + L.off_chunks);
  int* nchunks = (int*)(w + L.off_nchunks);
  int2* ranges = (int2*)(w + L.off_ranges);
  cudaStream_t st_ = (cudaStream_t)stream;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VQ2_ERR_NO_DEVICE;
  if (!g_pf_attr[dev]) {
    bool ok = true;
    ok &= cudaFuncSetAttribute(prefill_gemm_kernel<VQ2_PREC_FP8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P2_SMEM) == cudaSuccess;
    ok &= cudaFuncSetAttribute(prefill_gemm_kernel<VQ2_PREC_FP8, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P2_SMEM) == cudaSuccess;
    ok &= cudaFuncSetAttribute(prefill_gemm_kernel<VQ2_PREC_F16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P2_SMEM) == cudaSuccess;
    ok &= cudaFuncSetAttribute(prefill_gemm_kernel<VQ2_PREC_F16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)P2_SMEM) == cudaSuccess;
    if (!ok) return VQ2_ERR_CUDA;
    g_pf_attr[dev] = true;
  }
  const int nsm = device_sm_count();
  if (nsm <= 0) return VQ2_ERR_CUDA;
  int rc = launch_align_ex(a->topk_ids, a->ids_dtype, a->N, a->topk, a->E, P2_BM, a->expert_base, 1, st, ss, val,
                           be, counts, st_, ranges);
  if (rc) return rc;
  if (cudaMemsetAsync(a->out, 0, (size_t)a->N * a->H * sizeof(float), st_) != cudaSuccess) return VQ2_ERR_CUDA;
  build_chunks_kernel<<<1, 1024, 0, st_>>>(ranges, a->E, chunks, nchunks);

  P2Args g = {};
  g.chunks = chunks; g.nchunks = nchunks;
  g.st = st; g.ss = ss; g.val = val; g.topk_w = a->topk_w; g.inter = inter; g.out = a->out;
  g.I = a->I; g.H = a->H; g.topk = a->topk;
  if (prec == VQ2_PREC_FP8)
    had_quant_rows_kernel<VQ2_PREC_FP8><<<a->N, 256, 0, st_>>>(a->x, a->x_dtype, nullptr, a->H, xq, invx);
  else
    had_quant_rows_kernel<VQ2_PREC_F16><<<a->N, 256, 0, st_>>>(a->x, a->x_dtype, nullptr, a->H, xq, invx);
  const int elem = prec == VQ2_PREC_FP8 ? 1 : 2;
  const int lob = 128 / elem / 4;
  gather_slot_rows_kernel<<<(unsigned)L.Pmax, 256, 0, st_>>>(xq, invx, st, val, a->H * elem, xs, invxs);
  CUtensorMap tm_x, tm_v, tm_l13, tm_l2;
  if (encode_2d(&tm_x, xs, (uint64_t)a->H * elem, L.Pmax, 128, P2_NMAX, true) ||
      encode_2d(&tm_v, vb, (uint64_t)a->I * elem, L.Pmax, 128, P2_NMAX, true) ||
      encode_2d(&tm_l13, a->w13_lo, a->H / 4, (uint64_t)a->E * 2 * a->I, lob, P2_ROWS, false) ||
      encode_2d(&tm_l2, a->w2_lo, a->I / 4, (uint64_t)a->E * a->H, lob, P2_ROWS, false))
    return VQ2_ERR_CUDA;
  // gate/up: row tiles of 128 gate + 128 up rows
  g.inv_slot = invxs; g.lo = a->w13_lo; g.hi = a->w13_hi; g.sc = a->w13_sc; g.cb = a->w13_cb;
  g.K = a->H; g.R = 2 * a->I; g.T = a->I / P2_ROWS;
  if (prec == VQ2_PREC_FP8) prefill_gemm_kernel<VQ2_PREC_FP8, true><<<nsm, P2_THREADS, P2_SMEM, st_>>>(g, tm_x, tm_l13);
  else prefill_gemm_kernel<VQ2_PREC_F16, true><<<nsm, P2_THREADS, P2_SMEM, st_>>>(g, tm_x, tm_l13);
  // inter -> Hadamard -> quantised activation of the down projection
  if (prec == VQ2_PREC_FP8)
    had_quant_rows_kernel<VQ2_PREC_FP8><<<(unsigned)L.Pmax, 256, 0, st_>>>(inter, VQ2_DT_F32, val, a->I, vb, invvb);
  else
    had_quant_rows_kernel<VQ2_PREC_F16><<<(unsigned)L.Pmax, 256, 0, st_>>>(inter, VQ2_DT_F32, val, a->I, vb, invvb);
  // down + combine: row tiles of 256 output rows
  g.inv_slot = invvb; g.lo = a->w2_lo; g.hi = a->w2_hi; g.sc = a->w2_sc; g.cb = a->w2_cb;
  g.K = a->I; g.R = a->H; g.T = a->H / (P2_NT * P2_ROWS);
  if (prec == VQ2_PREC_FP8) prefill_gemm_kernel<VQ2_PREC_FP8, false><<<nsm, P2_THREADS, P2_SMEM, st_>>>(g, tm_v, tm_l2);
  else prefill_gemm_kernel<VQ2_PREC_F16, false><<<nsm, P2_THREADS, P2_SMEM, st_>>>(g, tm_v, tm_l2);
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}
