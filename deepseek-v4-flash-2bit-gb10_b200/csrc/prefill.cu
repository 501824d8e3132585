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
                    int32_t* ss, uint8_t* val, int32_t* be, int* counts, cudaStream_t stream);

constexpr int PF_BM = 128;            // slots per block (MMA M)
constexpr int PF_BN = 256;            // weight rows per tile (MMA N)
constexpr int PF_MB = 2;              // blocks of one expert sharing each decoded B tile
constexpr int PF_STAGES = 2;          // ring of A tiles (PF_MB blocks each): TMA from L2
constexpr int PF_ISTAGES = 3;         // ring of staged index planes: run ahead of the activations
constexpr int PF_BSTAGES = 2;         // ring of decoded B tiles: produced in the CTA
constexpr int PF_DEC_WARPS = 16;      // decoders; four per TMEM lane quarter in the epilogue
constexpr int PF_THREADS = (3 + PF_DEC_WARPS) * 32;   // A loader, index loader, MMA issuer, decoders
constexpr int PF_TILE = 16384;        // one 128-row x 128-byte activation tile
constexpr int PF_BTILE = PF_BN * 128; // the weight tile: 256 rows x 128 bytes
constexpr int PF_ATILE = PF_MB * PF_TILE;
constexpr int PF_CB_COPIES = 8;
constexpr int PF_CB_BYTES = 1024 * 8 * PF_CB_COPIES;
constexpr int PF_IDX = 11264;  // staged index planes of one stage: lo 8192 B, hi 2048 B, sc 1024 B
constexpr int PF_IDX_HI = 8192, PF_IDX_SC = 10240;
static_assert(PF_IDX % 16 == 0, "index stages keep 16-byte alignment");
constexpr int PF_TMEM_COLS = PF_MB * PF_BN;

struct PfShared {
  uint64_t full_a[PF_STAGES];
  uint64_t empty[PF_STAGES];
  uint64_t full_i[PF_ISTAGES];
  uint64_t empty_i[PF_ISTAGES];
  uint64_t full_b[PF_BSTAGES];
  uint64_t empty_b[PF_BSTAGES];
  uint64_t done[2];             // per pass: all MMAs of the pass complete
  uint64_t cbbar;
  uint32_t tmem_base;
};

constexpr size_t PF_SMEM = (size_t)PF_CB_BYTES + (size_t)PF_STAGES * PF_ATILE + (size_t)PF_ISTAGES * PF_IDX + (size_t)PF_BSTAGES * PF_BTILE +
                           sizeof(PfShared) + 1024;

struct PfGemmArgs {
  const uint8_t* act;        // activation rows (token rows for gate/up, slot rows for down)
  const float* inv_act;      // per activation row: inverse quantisation scale
  const int32_t* st;         // sorted_tok [Pmax]
  const int32_t* ss;         // sorted_slot [Pmax]
  const uint8_t* val;        // valid [Pmax]
  const int32_t* be;         // block -> local expert
  const uint8_t* lo;
  const uint8_t* hi;
  const uint16_t* sc;
  const uint16_t* cb;
  const float* topk_w;
  float* inter;              // gate/up output [Pmax, I]
  float* out;                // down output [N, H]
  int K;                     // input width (elements)
  int R;                     // weight rows per expert (2I or H)
  int I;
  int H;
  int topk;
};

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

// Instruction descriptor: D fp32, A/B format 0 (e4m3 for kind::f8f6f4, f16 for kind::f16),
// both K-major, N = 128, M = 128.
constexpr uint32_t PF_IDESC = (1u << 4) | ((uint32_t)(PF_BN >> 3) << 17) | ((uint32_t)(PF_BM >> 4) << 24);

template <int PREC>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t acc) {
  if (PREC == VQ2_PREC_FP8)
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n}"
                 ::"r"(tmem_d), "l"(da), "l"(db), "r"(PF_IDESC), "r"(acc));
  else
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
                 ::"r"(tmem_d), "l"(da), "l"(db), "r"(PF_IDESC), "r"(acc));
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

// byte offset of 16-byte chunk kc of row r in a 128 x 128-byte SW128 K-major tile
__device__ __forceinline__ uint32_t sw128_off(int r, int kc) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((kc ^ (r & 7)) << 4));
}

// ------------------------------------------------------------------ weight tile decode
// Decoder thread (row r, quarter h) fills 16-byte chunks 2h, 2h+1 of B row r of one stage:
// fp8: 8 sub-vectors -> 32 e4m3 values = e4m3(sat(C[id] * sc)) (reference vq2_grouped.cu:434-446);
// f16: 4 sub-vectors -> 16 f16 values C[id] * sc. lo: the sub-vectors' low bytes (little-endian
// in lo.x, lo.y); hw: their hi bits (2 per sub-vector from bit 0). cbl: this lane's codebook copy.
template <int PREC>
__device__ __forceinline__ void decode_b_quarter(uint32_t cbl, uint2 lo, uint32_t hw, float scf, uint32_t tile,
                                                 int r, int h) {
  if (PREC == VQ2_PREC_FP8) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {            // chunk 2h+q: sub-vectors 4q..4q+3
      uint32_t ids[2];
      unpack_ids4(q ? lo.y : lo.x, (hw >> (8 * q)) & 0xFFu, ids[0], ids[1]);
      uint32_t packed[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t id = (j & 2) ? (ids[j & 1] >> 16) : (ids[j & 1] & 0xFFFFu);
        const uint2 c = lds64(cbl + (id << 6));
        const float2 a = __half22float2(*(const __half2*)&c.x), b = __half22float2(*(const __half2*)&c.y);
        const __nv_fp8x2_storage_t p0 = __nv_cvt_float2_to_fp8x2(make_float2(a.x * scf, a.y * scf), __NV_SATFINITE, __NV_E4M3);
        const __nv_fp8x2_storage_t p1 = __nv_cvt_float2_to_fp8x2(make_float2(b.x * scf, b.y * scf), __NV_SATFINITE, __NV_E4M3);
        packed[j] = (uint32_t)p0 | ((uint32_t)p1 << 16);
      }
      sts128_v(tile + sw128_off(r, 2 * h + q), make_uint4(packed[0], packed[1], packed[2], packed[3]));
    }
  } else {
    const __half2 s2 = __float2half2_rn(scf);
    uint32_t ids[2];
    unpack_ids4(lo.x, hw & 0xFFu, ids[0], ids[1]);
#pragma unroll
    for (int q = 0; q < 2; ++q) {            // chunk 2h+q: sub-vectors 2q, 2q+1 (8 f16)
      uint32_t w[4];
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = 2 * q + jj;
        const uint32_t id = (j & 2) ? (ids[j & 1] >> 16) : (ids[j & 1] & 0xFFFFu);
        const uint2 c = lds64(cbl + (id << 6));
        const __half2 v0 = __hmul2(*(const __half2*)&c.x, s2), v1 = __hmul2(*(const __half2*)&c.y, s2);
        w[2 * jj] = *(const uint32_t*)&v0;
        w[2 * jj + 1] = *(const uint32_t*)&v1;
      }
      sts128_v(tile + sw128_off(r, 2 * h + q), make_uint4(w[0], w[1], w[2], w[3]));
    }
  }
}

// ------------------------------------------------------------------ grouped GEMM kernel
// grid (tiles along N, pairs of 128-slot blocks). GATEUP: tile n covers gate rows [128n, 128n+128)
// and the matching up rows; the epilogue writes inter. Otherwise tile n covers output rows
// [256n, 256n+256) and the epilogue accumulates into out. Two blocks of the same expert run as
// one pass (each decoded B tile feeds two MMAs, two TMEM accumulators); two blocks of different
// experts run as two passes, one accumulator each.

template <bool GATEUP>
__device__ __forceinline__ long pf_weight_row(const PfGemmArgs& a, int e, int tile, int r) {
  constexpr int HALF = PF_BN / 2;
  if (GATEUP) return (long)e * a.R + (r < HALF ? tile * HALF + r : a.I + tile * HALF + (r - HALF));
  return (long)e * a.R + tile * PF_BN + r;
}

struct PfPass {
  int blk;      // first block of the pass
  int mb;       // blocks in the pass (1 or 2)
  int e;        // local expert
  int acc;      // first TMEM accumulator
};

template <int PREC, bool GATEUP>
__global__ void __launch_bounds__(PF_THREADS, 1)
prefill_gemm_kernel(PfGemmArgs a, const __grid_constant__ CUtensorMap tm_act, const __grid_constant__ CUtensorMap tm_lo,
                    int nblk) {
  extern __shared__ __align__(1024) uint8_t pf_smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)pf_smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* cbs = smem;
  uint8_t* atiles = smem + PF_CB_BYTES;                // A ring (PF_MB tiles per stage)
  uint8_t* btiles = atiles + PF_STAGES * PF_ATILE;     // B ring
  uint8_t* itiles = btiles + PF_BSTAGES * PF_BTILE;    // index-plane ring
  PfShared* sh = (PfShared*)(itiles + PF_ISTAGES * PF_IDX);
  const int tile = blockIdx.x, b0 = blockIdx.y * PF_MB;
  if (!a.val[(size_t)b0 * PF_BM]) return;            // blocks past the last expert hold no pair
  const bool v1 = b0 + 1 < nblk && a.val[(size_t)(b0 + 1) * PF_BM];
  const int e0 = a.be[b0], e1 = v1 ? a.be[b0 + 1] : -1;
  // at most two passes, kept in registers (a run-time-indexed array would live in local memory)
  PfPass pass0, pass1 = {b0 + 1, 1, e1, 1};
  int npass;
  if (v1 && e1 == e0) { pass0 = {b0, 2, e0, 0}; npass = 1; }
  else if (v1) { pass0 = {b0, 1, e0, 0}; npass = 2; }
  else { pass0 = {b0, 1, e0, 0}; npass = 1; }
  auto pass_of = [&](int pi) { return pi == 0 ? pass0 : pass1; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int elem = PREC == VQ2_PREC_FP8 ? 1 : 2;
  constexpr int KE = 128 / elem;                      // K elements per stage (128 bytes per row)
  const int nchunks = a.K / KE;
  const int nsub = a.K / 4, ngk = a.K / 64;
  auto A_t = [&](int slot) { return atiles + slot * PF_ATILE; };
  auto B_t = [&](int slot) { return btiles + slot * PF_BTILE; };
  auto I_t = [&](int slot) { return itiles + slot * PF_IDX; };   // lo | hi | sc

  if (threadIdx.x == 0) {
    for (int s = 0; s < PF_STAGES; ++s) {
      mbar_init(&sh->full_a[s], 1);         // TMA bytes
      mbar_init(&sh->empty[s], 1);
    }
    for (int s = 0; s < PF_ISTAGES; ++s) {
      mbar_init(&sh->full_i[s], 33);        // TMA bytes (1 arrival) + 32 lanes' cp.async
      mbar_init(&sh->empty_i[s], PF_DEC_WARPS);
    }
    for (int s = 0; s < PF_BSTAGES; ++s) {
      mbar_init(&sh->full_b[s], PF_DEC_WARPS);
      mbar_init(&sh->empty_b[s], 1);
    }
    mbar_init(&sh->done[0], 1);
    mbar_init(&sh->done[1], 1);
    mbar_init(&sh->cbbar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&sh->cbbar, 1024 * 8);
    bulk_g2s(B_t(0), a.cb, 1024 * 8, &sh->cbbar);     // codebook lands in a B tile first
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&sh->tmem_base)), "r"(PF_TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  __syncthreads();                                    // barrier inits visible
  mbar_wait(&sh->cbbar, 0);
  {  // replicate: entry e of copy c at e*64 + c*8; consecutive 16-byte stores
    const uint2* src = (const uint2*)B_t(0);
    for (int idx = threadIdx.x; idx < 1024 * (PF_CB_COPIES / 2); idx += blockDim.x) {
      const uint2 v = src[idx / (PF_CB_COPIES / 2)];
      *(uint4*)(cbs + idx * 16) = make_uint4(v.x, v.y, v.x, v.y);
    }
  }
  tc_fence_before();
  __syncthreads();                                    // codebook ready, staging tile free again
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;

  if (warp == 0) {
    // ---------------- activation loader: A tiles of the pass's blocks by TMA (lane 0)
    if (lane == 0) {
      int gc = 0;
      for (int pi = 0; pi < npass; ++pi) {
        const PfPass P = pass_of(pi);
        for (int c = 0; c < nchunks; ++c, ++gc) {
          const int slot = gc % PF_STAGES;
          if (gc >= PF_STAGES && !mbar_wait(&sh->empty[slot], ((gc / PF_STAGES) - 1) & 1)) { pi = npass; break; }
          mbar_arrive_expect_tx(&sh->full_a[slot], P.mb * PF_TILE);
          tma_load_2d(A_t(slot), &tm_act, c * 128, P.blk * PF_BM, &sh->full_a[slot]);
          if (P.mb == 2) tma_load_2d(A_t(slot) + PF_TILE, &tm_act, c * 128, (P.blk + 1) * PF_BM, &sh->full_a[slot]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- index loader: lo plane by TMA, hi / scale planes by cp.async
    constexpr int LOB = 128 / elem / 4;               // lo bytes per row per stage (32 fp8, 16 f16)
    int gc = 0;
    for (int pi = 0; pi < npass; ++pi) {
      const PfPass P = pass_of(pi);
      const uint8_t* hi_r[8];
      const uint8_t* sc_r[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const long wr = pf_weight_row<GATEUP>(a, P.e, tile, lane + 32 * i);
        hi_r[i] = a.hi + wr * (nsub / 4);
        sc_r[i] = (const uint8_t*)(a.sc + wr * ngk);
      }
      const int row0 = (int)pf_weight_row<GATEUP>(a, P.e, tile, 0);
      const int row1 = (int)pf_weight_row<GATEUP>(a, P.e, tile, PF_BN / 2);
      for (int c = 0; c < nchunks; ++c, ++gc) {
        const int slot = gc % PF_ISTAGES;
        if (gc >= PF_ISTAGES && !mbar_wait(&sh->empty_i[slot], ((gc / PF_ISTAGES) - 1) & 1)) { pi = npass; break; }
        const uint32_t ibase = smem_u32(I_t(slot));
        if (lane == 0) {
          mbar_arrive_expect_tx(&sh->full_i[slot], PF_BN * LOB);
          tma_load_2d(I_t(slot), &tm_lo, c * LOB, row0, &sh->full_i[slot]);
          tma_load_2d(I_t(slot) + (PF_BN / 2) * LOB, &tm_lo, c * LOB, row1, &sh->full_i[slot]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = lane + 32 * i;
          if (PREC == VQ2_PREC_FP8) {          // hi: 8 bytes (32 sub-vectors); scales of 2 groups
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(ibase + PF_IDX_HI + r * 8), "l"(hi_r[i] + c * 8) : "memory");
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + PF_IDX_SC + r * 4), "l"(sc_r[i] + c * 4) : "memory");
          } else {                             // hi: 4 bytes (16 sub-vectors); the scale pair holding this group
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + PF_IDX_HI + r * 8), "l"(hi_r[i] + c * 4) : "memory");
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + PF_IDX_SC + r * 4), "l"(sc_r[i] + (c & ~1) * 2) : "memory");
          }
        }
        // one more arrival per lane when its copies above have landed
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&sh->full_i[slot])) : "memory");
      }
    }
    cp_async_wait<0>();                               // nothing in flight when the CTA retires
  } else if (warp == 2) {
    // ---------------- MMA issuer
    if (lane == 0) {
      int gc = 0;
      bool ok = true;
      for (int pi = 0; pi < npass && ok; ++pi) {
        const PfPass P = pass_of(pi);
        for (int c = 0; c < nchunks; ++c, ++gc) {
          const int slot = gc % PF_STAGES, bslot = gc % PF_BSTAGES;
          if (!mbar_wait(&sh->full_a[slot], (gc / PF_STAGES) & 1)) { ok = false; break; }
          if (!mbar_wait(&sh->full_b[bslot], (gc / PF_BSTAGES) & 1)) { ok = false; break; }
          fence_async_smem();                             // cp.async-written data visible to the tensor core
          tc_fence_after();
          const uint32_t abase = smem_u32(A_t(slot)), bbase = smem_u32(B_t(bslot));   // B: 256 rows
          for (int b = 0; b < P.mb; ++b) {
            const uint32_t td = tmem + (uint32_t)((P.acc + b) * PF_BN);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma<PREC>(td, umma_desc_sw128(abase + b * PF_TILE + ks * 32), umma_desc_sw128(bbase + ks * 32),
                         (c | ks) != 0);
          }
          umma_commit(&sh->empty[slot]);
          umma_commit(&sh->empty_b[bslot]);
        }
        umma_commit(&sh->done[pi]);   // arrives once every MMA issued so far has completed
      }
      for (int pi = 0; pi < npass; ++pi)
        if (!ok) umma_commit(&sh->done[pi]);          // let the epilogue finish (results invalid)
    }
  } else {
    // ---------------- weight decoders (512 threads: row r, half h of the 128-byte row)
    // the two half-row threads of a row are adjacent lanes: index-plane reads are contiguous
    const int dt = threadIdx.x - 96, r = dt >> 1, h = dt & 1;
    const uint32_t cbl = smem_u32(cbs + (lane & (PF_CB_COPIES - 1)) * 8);   // shared-window address
    int gc = 0;
    bool ok = true;
    for (int pi = 0; pi < npass; ++pi) {
      const PfPass P = pass_of(pi);
      for (int c = 0; c < nchunks && ok; ++c, ++gc) {
        const int slot = gc % PF_ISTAGES, bslot = gc % PF_BSTAGES;
        if (!mbar_wait(&sh->full_i[slot], (gc / PF_ISTAGES) & 1)) { ok = false; break; }
        if (gc >= PF_BSTAGES && !mbar_wait(&sh->empty_b[bslot], ((gc / PF_BSTAGES) - 1) & 1)) { ok = false; break; }
        const uint32_t ip = smem_u32(I_t(slot));
        const uint32_t bt = smem_u32(B_t(bslot));
        if (PREC == VQ2_PREC_FP8) {                   // 16 sub-vectors = one 64-group; lo rows 32 B apart
          const uint4 lo = lds128_v(ip + r * 32 + h * 16);
          const uint32_t hw = lds32_v(ip + PF_IDX_HI + r * 8 + h * 4);
          const uint32_t sbits = lds16_v(ip + PF_IDX_SC + r * 4 + h * 2);
          const float scf = __half2float(__ushort_as_half((unsigned short)sbits));
          decode_b_quarter<PREC>(cbl, make_uint2(lo.x, lo.y), hw & 0xFFFFu, scf, bt, r, 2 * h);
          decode_b_quarter<PREC>(cbl, make_uint2(lo.z, lo.w), hw >> 16, scf, bt, r, 2 * h + 1);
        } else {                                      // 8 sub-vectors; lo rows 16 B apart
          const uint2 lo = lds64_v(ip + r * 16 + h * 8);
          const uint32_t hw = lds16_v(ip + PF_IDX_HI + r * 8 + h * 2);
          const uint32_t sbits = lds16_v(ip + PF_IDX_SC + r * 4 + (c & 1) * 2);
          const float scf = __half2float(__ushort_as_half((unsigned short)sbits));
          decode_b_quarter<PREC>(cbl, make_uint2(lo.x, 0u), hw & 0xFFu, scf, bt, r, 2 * h);
          decode_b_quarter<PREC>(cbl, make_uint2(lo.y, 0u), hw >> 8, scf, bt, r, 2 * h + 1);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sh->full_b[bslot]);
          mbar_arrive(&sh->empty_i[slot]);
        }
      }
      // ---------------- epilogue of the pass out of TMEM
      const int q = warp & 3, cq = (warp - 3) >> 2;        // TMEM lane quarter, column quarter
      if (!mbar_wait(&sh->done[pi], 0)) continue;
      tc_fence_after();
      for (int b = 0; b < P.mb; ++b) {
        const int slot_i = q * 32 + lane;
        const size_t p = (size_t)(P.blk + b) * PF_BM + slot_i;
        const int tok = a.val[p] ? a.st[p] : -1;
        const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((P.acc + b) * PF_BN);
        if (GATEUP) {                                  // 32 gate + the 32 matching up columns
          float g[32], u[32];
          tmem_ld32(trow + cq * 32, g);
          tmem_ld32(trow + PF_BN / 2 + cq * 32, u);
          const float inv = tok >= 0 ? a.inv_act[tok] : 0.f;
          float* dst = a.inter + p * a.I + tile * (PF_BN / 2) + cq * 32;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            float rr[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const float gg = g[j + t] * inv, uu = u[j + t] * inv;
              rr[t] = gg / (1.f + __expf(-gg)) * uu;
            }
            *(float4*)(dst + j) = make_float4(rr[0], rr[1], rr[2], rr[3]);
          }
        } else {                                       // 64 output columns
          const float w = tok >= 0 ? a.topk_w[(size_t)tok * a.topk + a.ss[p]] * a.inv_act[p] : 0.f;
          float* dst = a.out + (size_t)(tok >= 0 ? tok : 0) * a.H + tile * PF_BN + cq * 64;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float v[32];
            tmem_ld32(trow + cq * 64 + hh * 32, v);     // collective: every lane loads
            if (tok >= 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                atomicAdd((float4*)(dst + hh * 32 + j), make_float4(v[j] * w, v[j + 1] * w, v[j + 2] * w, v[j + 3] * w));
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PF_TMEM_COLS) : "memory");
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

// Quantised token rows into slot order (padding slots zero), so the gate/up A tile of a block is
// one contiguous 2-D TMA box.
__global__ void __launch_bounds__(256) gather_slot_rows_kernel(const uint8_t* __restrict__ src,
                                                              const int32_t* __restrict__ st,
                                                              const uint8_t* __restrict__ val, int row_bytes,
                                                              uint8_t* __restrict__ dst) {
  const long p = blockIdx.x;
  uint4* d = (uint4*)(dst + p * (size_t)row_bytes);
  const bool ok = val[p] != 0;
  const uint4* s = (const uint4*)(src + (size_t)(ok ? st[p] : 0) * row_bytes);
  for (int i = threadIdx.x; i < row_bytes / 16; i += blockDim.x) d[i] = ok ? s[i] : make_uint4(0, 0, 0, 0);
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
  long M, Pmax, nblk, nchunks;
  size_t off_st, off_ss, off_val, off_be, off_counts, off_xq, off_invx, off_xs, off_inter, off_vb, off_invvb, total;
};

static size_t up256(size_t v) { return (v + 255) & ~(size_t)255; }

static PfLayout pf_layout(int N, int k, int E, int H, int I, int prec) {
  PfLayout L;
  const size_t elem = prec == VQ2_PREC_FP8 ? 1 : 2;
  L.M = (long)N * k;
  L.Pmax = L.M + (long)std::min<long>(L.M, E) * PF_BM;
  L.nblk = L.Pmax / PF_BM;
  L.nchunks = std::max<long>(1, (L.M + 8191) / 8192);
  size_t o = 0;
  L.off_st = o; o = up256(o + L.Pmax * 4);
  L.off_ss = o; o = up256(o + L.Pmax * 4);
  L.off_val = o; o = up256(o + L.Pmax);
  L.off_be = o; o = up256(o + L.nblk * 4);
  L.off_counts = o; o = up256(o + L.nchunks * E * 4);
  L.off_xq = o; o = up256(o + (size_t)N * H * elem);
  L.off_invx = o; o = up256(o + (size_t)N * 4);
  L.off_xs = o; o = up256(o + (size_t)L.Pmax * H * elem);
  L.off_inter = o; o = up256(o + (size_t)L.Pmax * I * 4);
  L.off_vb = o; o = up256(o + (size_t)L.Pmax * I * elem);
  L.off_invvb = o; o = up256(o + (size_t)L.Pmax * 4);
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
  if (L.nblk > 65535) return VQ2_ERR_SHAPE;
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
  float* inter = (float*)(w + L.off_inter);
  uint8_t* vb = w + L.off_vb;
  float* invvb = (float*)(w + L.off_invvb);
  cudaStream_t st_ = (cudaStream_t)stream;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return VQ2_ERR_NO_DEVICE;
  if (!g_pf_attr[dev]) {
    bool ok = true;
    ok &= cudaFuncSetAttribute(prefill_gemm_kernel<VQ2_PREC_FP8, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM) == cudaSuccess;
    ok &= cudaFuncSetAttribute(prefill_gemm_kernel<VQ2_PREC_FP8, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM) == cudaSuccess;
    ok &= cudaFuncSetAttribute(prefill_gemm_kernel<VQ2_PREC_F16, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM) == cudaSuccess;
    ok &= cudaFuncSetAttribute(prefill_gemm_kernel<VQ2_PREC_F16, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM) == cudaSuccess;
    if (!ok) return VQ2_ERR_CUDA;
    g_pf_attr[dev] = true;
  }
  int rc = launch_align_ex(a->topk_ids, a->ids_dtype, a->N, a->topk, a->E, PF_BM, a->expert_base, 1, st, ss, val,
                           be, counts, st_);
  if (rc) return rc;
  if (cudaMemsetAsync(a->out, 0, (size_t)a->N * a->H * sizeof(float), st_) != cudaSuccess) return VQ2_ERR_CUDA;

  PfGemmArgs g = {};
  g.act = nullptr;
  g.st = st; g.ss = ss; g.val = val; g.be = be; g.topk_w = a->topk_w; g.inter = inter; g.out = a->out;
  g.I = a->I; g.H = a->H; g.topk = a->topk;
  if (prec == VQ2_PREC_FP8) {
    had_quant_rows_kernel<VQ2_PREC_FP8><<<a->N, 256, 0, st_>>>(a->x, a->x_dtype, nullptr, a->H, xq, invx);
  } else {
    had_quant_rows_kernel<VQ2_PREC_F16><<<a->N, 256, 0, st_>>>(a->x, a->x_dtype, nullptr, a->H, xq, invx);
  }
  const int elem = prec == VQ2_PREC_FP8 ? 1 : 2;
  const int lob = 128 / elem / 4;
  gather_slot_rows_kernel<<<(unsigned)L.Pmax, 256, 0, st_>>>(xq, st, val, a->H * elem, xs);
  CUtensorMap tm_x, tm_v, tm_l13, tm_l2;
  if (encode_2d(&tm_x, xs, (uint64_t)a->H * elem, L.Pmax, 128, 128, true) ||
      encode_2d(&tm_v, vb, (uint64_t)a->I * elem, L.Pmax, 128, 128, true) ||
      encode_2d(&tm_l13, a->w13_lo, a->H / 4, (uint64_t)a->E * 2 * a->I, lob, PF_BN / 2, false) ||
      encode_2d(&tm_l2, a->w2_lo, a->I / 4, (uint64_t)a->E * a->H, lob, PF_BN / 2, false))
    return VQ2_ERR_CUDA;
  // gate/up
  g.inv_act = invx; g.lo = a->w13_lo; g.hi = a->w13_hi; g.sc = a->w13_sc; g.cb = a->w13_cb;
  g.K = a->H; g.R = 2 * a->I;
  dim3 g1(a->I / (PF_BN / 2), (unsigned)((L.nblk + PF_MB - 1) / PF_MB));
  if (prec == VQ2_PREC_FP8) prefill_gemm_kernel<VQ2_PREC_FP8, true><<<g1, PF_THREADS, PF_SMEM, st_>>>(g, tm_x, tm_l13, (int)L.nblk);
  else prefill_gemm_kernel<VQ2_PREC_F16, true><<<g1, PF_THREADS, PF_SMEM, st_>>>(g, tm_x, tm_l13, (int)L.nblk);
  // inter -> Hadamard -> quantised activation of the down projection
  if (prec == VQ2_PREC_FP8)
    had_quant_rows_kernel<VQ2_PREC_FP8><<<(unsigned)L.Pmax, 256, 0, st_>>>(inter, VQ2_DT_F32, val, a->I, vb, invvb);
  else
    had_quant_rows_kernel<VQ2_PREC_F16><<<(unsigned)L.Pmax, 256, 0, st_>>>(inter, VQ2_DT_F32, val, a->I, vb, invvb);
  // down + combine
  g.inv_act = invvb; g.lo = a->w2_lo; g.hi = a->w2_hi; g.sc = a->w2_sc; g.cb = a->w2_cb;
  g.K = a->I; g.R = a->H;
  dim3 g2(a->H / PF_BN, (unsigned)((L.nblk + PF_MB - 1) / PF_MB));
  if (prec == VQ2_PREC_FP8) prefill_gemm_kernel<VQ2_PREC_FP8, false><<<g2, PF_THREADS, PF_SMEM, st_>>>(g, tm_v, tm_l2, (int)L.nblk);
  else prefill_gemm_kernel<VQ2_PREC_F16, false><<<g2, PF_THREADS, PF_SMEM, st_>>>(g, tm_v, tm_l2, (int)L.nblk);
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}
