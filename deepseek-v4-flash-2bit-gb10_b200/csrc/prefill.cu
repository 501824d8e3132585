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

// fp8 from an fp32 codebook (entries 128 bytes apart: 8 copies of 16 bytes, lane l reads copy
// l mod 8, so each 8-lane phase of a warp's 16-byte gathers is conflict-free): one gather gives
// the four fp32 values, two packed multiplies give the exact products, then e4m3 as above.
__device__ __forceinline__ void decode8_fp8_f32cb(uint32_t cbl, uint2 lo, uint32_t hw, float scf, uint32_t* v) {
  const float2 s2 = make_float2(scf, scf);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint32_t ids[2];
    unpack_ids4(q ? lo.y : lo.x, (hw >> (8 * q)) & 0xFFu, ids[0], ids[1]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t id = (j & 2) ? (ids[j & 1] >> 16) : (ids[j & 1] & 0xFFFFu);
      float4 c;
      asm("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(c.x), "=f"(c.y), "=f"(c.z), "=f"(c.w) : "r"(cbl + (id << 7)));
      const __nv_fp8x2_storage_t p0 = __nv_cvt_float2_to_fp8x2(fmul2(make_float2(c.x, c.y), s2), __NV_SATFINITE, __NV_E4M3);
      const __nv_fp8x2_storage_t p1 = __nv_cvt_float2_to_fp8x2(fmul2(make_float2(c.z, c.w), s2), __NV_SATFINITE, __NV_E4M3);
      v[4 * q + j] = (uint32_t)p0 | ((uint32_t)p1 << 16);
    }
  }
}

// f16: 4 sub-vectors of a row (lo: 4 low index bytes, hw: 1 hi byte) -> 8 words of 2 f16 values,
// C[id] * sc in fp16.
__device__ __forceinline__ void decode4_f16(uint32_t cbl, uint32_t lo, uint32_t hw, unsigned short sb, uint32_t* v) {
  const __half2 s2 = __half2half2(__ushort_as_half(sb));
  uint32_t h02, h13;
  ids_hi_pairs(hw & 0xFFu, h02, h13);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t id = j == 0 ? id_of<0>(lo, h02, h13) : j == 1 ? id_of<1>(lo, h02, h13)
                      : j == 2 ? id_of<2>(lo, h02, h13) : id_of<3>(lo, h02, h13);
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

// ------------------------------------------------------------------ grouped GEMM kernel (CTA pairs)
// Persistent; the CTAs run as pairs (clusters of 2) and pair p walks the work list
// w = p, p + npairs, ... (w -> chunk w / T, row tile w % T; chunks heaviest first). A work item is
// one chunk of up to P2_NMAX consecutive slots of one expert (its tokens, padded to P2_BM) against
// 256 weight rows: 128 per CTA of the pair (GATEUP: 64 gate rows and the 64 matching up rows of
// the pair's 128 intermediate columns; otherwise 128 down rows). Per 128-byte K stage each CTA's
// decoder warps write its 128 decoded rows into its tensor memory (the A operand, M = 256 over the
// pair), each CTA loads half of the slots of every accumulator by TMA (the B operand, N split over
// the pair), and the first CTA's MMA lane issues cta_group::2 MMAs (M = 256, N <= 192) into two
// accumulators per CTA (up to 384 slots per item). The pair shares every activation tile, so the
// activation traffic per weight row is half that of one CTA holding 256 rows, and each decoded
// weight serves up to 384 slots. The epilogue reads each CTA's accumulators (lane = weight row,
// column = slot): gate/up pairs the gate and up lanes (adjacent lanes) by shuffles and writes
// inter[slot][i] = silu(g * inv) * (u * inv) (reference vq2_grouped.cu:255-264); down adds
// acc * w * inv_vb into out[token] with fp32 reductions.
constexpr int P2_ROWS = 128;                 // weight rows per CTA (half of the pair's MMA M)
constexpr int P2_NACC = 2;                   // accumulators per CTA
constexpr int P2_NSUB = 192;                 // slots per accumulator (MMA N at most)
constexpr int P2_NMAX = P2_NACC * P2_NSUB;   // slots per chunk
constexpr int P2_BM = 32;                    // per-expert slot padding (moe_align block)
constexpr int P2_CHUNK_BLOCKS = P2_NMAX / P2_BM;
constexpr int P2_BSTAGES = 3, P2_ISTAGES = 4, P2_ASTAGES = 4;
constexpr int P2_DEC_WARPS = 16;             // 4 per TMEM lane quarter: K quarter
constexpr int P2_THREADS = (3 + P2_DEC_WARPS) * 32;
constexpr int P2_BHALF = (P2_NSUB / 2) * 128;          // one CTA's half of one accumulator's B: 96 rows
constexpr int P2_BTILE = P2_NACC * P2_BHALF;           // one B stage of one CTA
constexpr int P2_CB_COPIES = 16;
constexpr int P2_CB_BYTES = 1024 * 8 * P2_CB_COPIES;
constexpr int P2_IDX = 5632;                 // index planes of one stage: lo [LOB/16][128][16], hi 128 x 8, sc 128 x 4
constexpr int P2_IDX_HI = 4096, P2_IDX_SC = 5120;
constexpr uint32_t P2_TMEM_COLS = 512;
// TMEM columns: accumulator 0 at 0 (N <= 192), A stages 0-1 at 192 and 224, accumulator 1 at 256,
// A stages 2-3 at 448 and 480 (32 columns each: 128 bytes of K).
__host__ __device__ constexpr uint32_t p2_acc_col(int j) { return j ? 256u : 0u; }
__host__ __device__ constexpr uint32_t p2_a_col(int s) { return s < 2 ? 192u + 32u * s : 448u + 32u * (s - 2); }

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
  int T;                     // row tiles (pair items) per chunk
};

// ---- cluster-pair helpers
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the address of this CTA's shared variable `p` in CTA `cta` of the cluster
__device__ __forceinline__ uint32_t peer_smem(const void* p, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(cta));
  return r;
}
// Arrive on a barrier of another CTA of the cluster (default release semantics at CTA scope;
// tensor-memory writes are ordered by the tcgen05 fences around the barrier, as the pair leader's
// MMA lane issues tcgen05.fence::after_thread_sync after its wait).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (for barriers the peer CTA arrives on).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < VQ2_WAIT_LIMIT; ++i)
    if (mbar_try_wait_cluster(bar, parity)) return true;
  set_status(VQ2_ERR_TIMEOUT);
  return false;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 2-D TMA load into this CTA's shared memory whose completion is counted on the pair leader's
// barrier (`bar_cluster`: a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
               ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(bar_cluster) : "memory");
}
template <int PREC>
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
  if (PREC == VQ2_PREC_FP8)
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], [%1], %2, %3, p;\n}"
                 ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
  else
    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                 " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}"
                 ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc));
}
// arrives on the barrier at this offset in both CTAs once every prior MMA of the pair completed
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               ::"r"(smem_u32(bar)), "h"((unsigned short)3) : "memory");
}

// Weight row of row R (0..127) of this CTA's index stage in pair item `tile` of expert e (rank:
// the CTA in the pair). GATEUP: R < 64 are the gate rows of the CTA's 64 intermediate columns,
// R >= 64 the matching up rows; otherwise 128 consecutive down rows.
template <bool GATEUP>
__device__ __forceinline__ long p2_weight_row(const P2Args& a, int e, int tile, int rank, int R) {
  if (GATEUP) {
    const int i = tile * P2_ROWS + rank * (P2_ROWS / 2) + (R & 63);     // intermediate column
    return (long)e * a.R + (R < 64 ? i : a.I + i);
  }
  return (long)e * a.R + (long)tile * (2 * P2_ROWS) + rank * P2_ROWS + R;
}
// Index-stage row decoded into TMEM lane r. GATEUP interleaves gate and up: lane 2m holds the gate
// row and lane 2m + 1 the up row of intermediate column m, so the epilogue pairs them with a lane
// shuffle.
template <bool GATEUP>
__device__ __forceinline__ int p2_stage_row(int r) { return GATEUP ? (r & 1) * 64 + (r >> 1) : r; }

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
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
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
    for (int s = 0; s < P2_ASTAGES; ++s) { mbar_init(&sh->full_a[s], 2 * P2_DEC_WARPS); mbar_init(&sh->empty_a[s], 1); }
    mbar_init(&sh->done, 1);
    mbar_init(&sh->acc_empty, 2 * P2_DEC_WARPS);
    mbar_init(&sh->cbbar, 1);
    mbar_init(&sh->drain, 1);
    sh->abort = 0;
    fence_mbar_init();
    mbar_arrive_expect_tx(&sh->cbbar, 1024 * 8);
    bulk_g2s(B_t(0), a.cb, 1024 * 8, &sh->cbbar);     // the codebook lands in a B stage first
  }
  if (warp == 0) {   // the same warp in both CTAs of the pair (a collective allocation)
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&sh->tmem_base)), "r"(P2_TMEM_COLS) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  __syncthreads();
  if (!mbar_wait(&sh->cbbar, 0)) sh->abort = 1;
  if (PREC == VQ2_PREC_FP8) {  // fp32 entries: entry e of copy c at e * 128 + c * 16
    const uint2* src = (const uint2*)B_t(0);
    for (int idx = threadIdx.x; idx < 1024 * 8; idx += blockDim.x) {
      const uint2 v = src[idx >> 3];
      const float2 a = __half22float2(*(const __half2*)&v.x), b = __half22float2(*(const __half2*)&v.y);
      *(float4*)(cbs + idx * 16) = make_float4(a.x, a.y, b.x, b.y);
    }
  } else {  // fp16 entries: entry e of copy c at e * 128 + c * 8; consecutive 16-byte stores
    const uint2* src = (const uint2*)B_t(0);
    for (int idx = threadIdx.x; idx < 1024 * (P2_CB_COPIES / 2); idx += blockDim.x) {
      const uint2 v = src[idx / (P2_CB_COPIES / 2)];
      *(uint4*)(cbs + idx * 16) = make_uint4(v.x, v.y, v.x, v.y);
    }
  }
  tc_fence_before();
  __syncthreads();                                     // codebook ready, B stage 0 free again
  cluster_sync();                                      // both CTAs' barriers initialised
  tc_fence_after();
  const uint32_t tmem = sh->tmem_base;
  volatile int* abort = &sh->abort;

  if (warp == 0) {
    // ---------------- activation loader (lane 0): this CTA's halves of the item's B stages
    if (lane == 0) {
      int gb = 0;
      for (int w = pair; w < nwork && !*abort; w += npairs) {
        const int4 ch = a.chunks[w / a.T];
        const int n0 = min(ch.z, P2_NSUB), n1 = ch.z - n0;     // slots of the two accumulators
        const int nacc = n1 > 0 ? 2 : 1;
        for (int c = 0; c < nstage; ++c, ++gb) {
          const int slot = gb % P2_BSTAGES;
          if (gb >= P2_BSTAGES && !mbar_wait(&sh->empty_b[slot], ((gb / P2_BSTAGES) - 1) & 1)) { *abort = 1; break; }
          const uint32_t fb = peer_smem(&sh->full_b[slot], 0);
          if (leader) mbar_arrive_expect_tx(&sh->full_b[slot], 2u * nacc * P2_BHALF);
          tma_load_2d_pair(B_t(slot), &tm_act, c * 128, ch.y + (int)rank * (n0 >> 1), fb);
          if (nacc == 2) tma_load_2d_pair(B_t(slot) + P2_BHALF, &tm_act, c * 128, ch.y + P2_NSUB + (int)rank * (n1 >> 1), fb);
        }
      }
      // both CTAs' loads of the last stages complete on the leader's barriers: the leader waits
      // for them (bounded) so no copy is in flight when the pair exits
      if (leader)
        for (int q = max(0, gb - P2_BSTAGES); q < gb; ++q) mbar_wait_cluster(&sh->full_b[q % P2_BSTAGES], (q / P2_BSTAGES) & 1);
    }
  } else if (warp == 1) {
    // ---------------- index loader: lo plane by TMA (two 64-row boxes), hi / scale planes by cp.async
    int gi = 0;
    for (int w = pair; w < nwork && !*abort; w += npairs) {
      const int e = a.chunks[w / a.T].x, tile = w % a.T;
      const int row0 = (int)p2_weight_row<GATEUP>(a, e, tile, rank, 0);
      const int row1 = (int)p2_weight_row<GATEUP>(a, e, tile, rank, 64);
      const uint8_t* hi_r[4];
      const uint8_t* sc_r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const long wr = p2_weight_row<GATEUP>(a, e, tile, rank, lane + 32 * i);
        hi_r[i] = a.hi + wr * (nsub / 4);
        sc_r[i] = (const uint8_t*)(a.sc + wr * ngk);
      }
      for (int c = 0; c < nstage; ++c, ++gi) {
        const int slot = gi % P2_ISTAGES;
        if (gi >= P2_ISTAGES && !mbar_wait(&sh->empty_i[slot], ((gi / P2_ISTAGES) - 1) & 1)) { *abort = 1; break; }
        const uint32_t ibase = smem_u32(I_t(slot));
        if (lane == 0) {
          mbar_arrive_expect_tx(&sh->full_i[slot], P2_ROWS * LOB);
          // 16-byte-wide boxes: [16-byte column h][row 0..127][16 bytes] (fp8: two columns), so a
          // decoder warp's 8-byte reads of 32 rows stride 16 bytes instead of LOB
#pragma unroll
          for (int h = 0; h < LOB / 16; ++h) {
            tma_load_2d(I_t(slot) + h * (P2_ROWS * 16), &tm_lo, c * LOB + h * 16, row0, &sh->full_i[slot]);
            tma_load_2d(I_t(slot) + h * (P2_ROWS * 16) + 64 * 16, &tm_lo, c * LOB + h * 16, row1, &sh->full_i[slot]);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int R = lane + 32 * i;
          if (PREC == VQ2_PREC_FP8) {          // hi: 8 bytes (32 sub-vectors); scales of 2 groups
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(ibase + P2_IDX_HI + R * 8), "l"(hi_r[i] + c * 8) : "memory");
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + P2_IDX_SC + R * 4), "l"(sc_r[i] + c * 4) : "memory");
          } else {                             // hi: 4 bytes (16 sub-vectors); the scale pair holding this group
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + P2_IDX_HI + R * 8), "l"(hi_r[i] + c * 4) : "memory");
            asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(ibase + P2_IDX_SC + R * 4), "l"(sc_r[i] + (c & ~1) * 2) : "memory");
          }
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&sh->full_i[slot])) : "memory");
      }
    }
    cp_async_wait<0>();
    if (lane == 0)   // the lo-plane TMA loads of the last stages have landed
      for (int q = max(0, gi - P2_ISTAGES); q < gi; ++q) mbar_wait(&sh->full_i[q % P2_ISTAGES], (q / P2_ISTAGES) & 1);
  } else if (warp == 2) {
    // ---------------- MMA issuer (lane 0 of the pair's first CTA)
    if (lane == 0 && leader) {
      int gb = 0, ga = 0, it = 0;
      for (int w = pair; w < nwork && !*abort; w += npairs, ++it) {
        const int ns = a.chunks[w / a.T].z;
        const int n0 = min(ns, P2_NSUB), n1 = ns - n0;
        const uint32_t id0 = (1u << 4) | ((uint32_t)(n0 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
        const uint32_t id1 = (1u << 4) | ((uint32_t)(n1 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
        if (it > 0 && !mbar_wait_cluster(&sh->acc_empty, (it - 1) & 1)) { *abort = 1; break; }
        tc_fence_after();
        bool ok = true;
        for (int c = 0; c < nstage; ++c, ++gb, ++ga) {
          const int bslot = gb % P2_BSTAGES, aslot = ga % P2_ASTAGES;
          if (!mbar_wait_cluster(&sh->full_b[bslot], (gb / P2_BSTAGES) & 1) ||
              !mbar_wait_cluster(&sh->full_a[aslot], (ga / P2_ASTAGES) & 1)) { ok = false; break; }
          tc_fence_after();
          const uint32_t bbase = smem_u32(B_t(bslot));
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_pair<PREC>(tmem + p2_acc_col(0), tmem + p2_a_col(aslot) + 8 * ks, umma_desc_sw128(bbase + ks * 32), id0,
                            (c | ks) != 0);
          if (n1 > 0) {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_pair<PREC>(tmem + p2_acc_col(1), tmem + p2_a_col(aslot) + 8 * ks,
                              umma_desc_sw128(bbase + P2_BHALF + ks * 32), id1, (c | ks) != 0);
          }
          umma_commit_pair(&sh->empty_b[bslot]);
          umma_commit_pair(&sh->empty_a[aslot]);
        }
        umma_commit_pair(&sh->done);   // both CTAs: every MMA issued so far has completed
        if (!ok) { *abort = 1; break; }
      }
      umma_commit_pair(&sh->drain);    // nothing of ours still reads TMEM or shared memory after this
      mbar_wait(&sh->drain, 0);
    }
  } else {
    // ---------------- decoders (16 warps): warp -> TMEM lane quarter q, K quarter kq
    // Software-pipelined by one stage: the tensor-memory store of stage c is issued, then stage
    // c + 1's index planes are read and decoded into registers, and only then is the store of
    // stage c waited for and the stage handed to the MMA lane (the pair leader's barrier), so
    // the store latency does not sit on the decode chain.
    const int q = warp & 3, kq = (warp - 3) >> 2;
    const int r = q * 32 + lane;                           // TMEM lane
    const int R = p2_stage_row<GATEUP>(r);                 // its row of the index stage
    const uint32_t cbl = PREC == VQ2_PREC_FP8 ? smem_u32(cbs) + (lane & 7) * 16      // fp32 codebook: 8 copies
                                              : smem_u32(cbs) + (lane & (P2_CB_COPIES - 1)) * 8;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    int gi = 0, ga = 0, it = 0;
    // stage gi of the index ring -> 8 decoded words (this thread's row, K quarter), then frees
    // the slot (after the decode consumed every lane's loads of it: the next writer is the
    // loader's TMA / cp.async)
    auto decode_stage = [&](int c, uint32_t* v) -> bool {
      const int islot = gi % P2_ISTAGES;
      if (!mbar_wait(&sh->full_i[islot], (gi / P2_ISTAGES) & 1)) return false;
      const uint32_t ip = smem_u32(I_t(islot));
      if (PREC == VQ2_PREC_FP8) {             // 8 sub-vectors, a quarter of the 128-element stage
        const uint2 lo = lds64_v(ip + (kq >> 1) * (P2_ROWS * 16) + R * 16 + (kq & 1) * 8);
        const uint32_t hw = lds16_v(ip + P2_IDX_HI + R * 8 + kq * 2);
        const uint32_t sbits = lds16_v(ip + P2_IDX_SC + R * 4 + (kq >> 1) * 2);
        decode8_fp8_f32cb(cbl, lo, hw, __half2float(__ushort_as_half((unsigned short)sbits)), v);
      } else {                                // 4 sub-vectors, a quarter of the 64-element stage
        const uint32_t lo = lds32_v(ip + R * 16 + kq * 4);
        const uint32_t hw = lds8_v(ip + P2_IDX_HI + R * 8 + kq);
        const uint32_t sbits = lds16_v(ip + P2_IDX_SC + R * 4 + (c & 1) * 2);
        decode4_f16(cbl, lo, hw, (unsigned short)sbits, v);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty_i[islot]);
      ++gi;
      return true;
    };
    const uint32_t full_a0 = peer_smem(&sh->full_a[0], 0), acc_empty0 = peer_smem(&sh->acc_empty, 0);
    const uint32_t full_a_step = (uint32_t)((uintptr_t)&sh->full_a[1] - (uintptr_t)&sh->full_a[0]);
    for (int w = pair; w < nwork; w += npairs, ++it) {
      const int4 ch = a.chunks[w / a.T];
      const int tile = w % a.T;
      bool ok = !*abort;
      // two register sets: a tcgen05.st reads its source registers asynchronously, so the set
      // being stored stays untouched (and is kept live) until its tcgen05.wait::st
      uint32_t va[8], vb[8];
      if (ok) ok = decode_stage(0, va);
      auto step = [&](int c, uint32_t* cur, uint32_t* nxt) {
        const int aslot = ga % P2_ASTAGES;
        if (ga >= P2_ASTAGES && !mbar_wait(&sh->empty_a[aslot], ((ga / P2_ASTAGES) - 1) & 1)) { ok = false; return; }
        tc_fence_after();
        tmem_st8(tmem + tlane + p2_a_col(aslot) + 8 * kq, cur);
        if (c + 1 < nstage && !decode_stage(c + 1, nxt)) ok = false;
        tmem_st_wait();
        keep_live8(cur);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(full_a0 + aslot * full_a_step);
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
      const int n0 = min(ch.z, P2_NSUB);
      const int ncol = ch.z >> 5;                           // 32-slot column groups over both accumulators
      if (GATEUP) {
        // lane 2m holds gate and lane 2m + 1 up of intermediate column m; for each column pair
        // (k, k + 1) the even lane finishes slot k and the odd lane slot k + 1
        const bool odd = lane & 1;
        float* dst = a.inter + tile * P2_ROWS + rank * (P2_ROWS / 2) + (r >> 1);
        for (int cg = kq; cg < ncol; cg += 4) {
          const int j = cg * 32 >= n0 ? 1 : 0;
          const int col = cg * 32 - j * P2_NSUB;             // column within accumulator j
          const int s0 = ch.y + j * P2_NSUB + col;           // slot of that column
          const float myinv = a.inv_slot[s0 + lane];
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            float v[16];
            tmem_ld16(tmem + tlane + p2_acc_col(j) + col + hh * 16, v);
#pragma unroll
            for (int k = 0; k < 16; k += 2) {
              // even lane keeps column k, odd lane column k + 1; each sends the other column
              const float send = odd ? v[k] : v[k + 1];
              const float recv = __shfl_xor_sync(0xffffffffu, send, 1);
              const float g = odd ? recv : v[k], u = odd ? v[k + 1] : recv;
              const int kk = hh * 16 + k + (odd ? 1 : 0);
              const float inv = __shfl_sync(0xffffffffu, myinv, kk);
              const float gg = g * inv, uu = u * inv;
              dst[(size_t)(s0 + kk) * a.I] = __fdividef(gg, 1.f + __expf(-gg)) * uu;
            }
          }
        }
      } else {
        float* col_out = a.out + tile * (2 * P2_ROWS) + rank * P2_ROWS + r;
        for (int cg = kq; cg < ncol; cg += 4) {
          const int j = cg * 32 >= n0 ? 1 : 0;
          const int col = cg * 32 - j * P2_NSUB;
          const int s = ch.y + j * P2_NSUB + col + lane;
          const int mytok = a.val[s] ? a.st[s] : -1;
          const float myw = mytok >= 0 ? a.topk_w[(size_t)mytok * a.topk + a.ss[s]] * a.inv_slot[s] : 0.f;
#pragma unroll 1
          for (int hh = 0; hh < 2; ++hh) {
            float v[16];
            tmem_ld16(tmem + tlane + p2_acc_col(j) + col + hh * 16, v);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const int tok = __shfl_sync(0xffffffffu, mytok, hh * 16 + k);
              const float wk = __shfl_sync(0xffffffffu, myw, hh * 16 + k);
              if (tok >= 0) atomicAdd(col_out + (size_t)tok * a.H, v[k] * wk);   // 32 consecutive rows: one line
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc_empty0);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();                                      // the pair's MMAs and TMEM reads are done
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P2_TMEM_COLS) : "memory");
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
// Rows with valid[row] == 0 are written as zeros with inv = 0. cols <= 4096. With `pslot`, row n
// is a token whose quantised row (and inverse scale) is written to each of its slots
// pslot[n * k + j] >= 0 instead of row n of `out` (the slot gather fused into the quantisation).
template <int PREC>
__global__ void __launch_bounds__(256) had_quant_rows_kernel(const void* __restrict__ x, int in_dt,
                                                             const uint8_t* __restrict__ valid, int cols,
                                                             uint8_t* __restrict__ out, float* __restrict__ inv,
                                                             const int32_t* __restrict__ pslot, int k) {
  __shared__ float red[33];
  __shared__ __align__(16) uint8_t qrow[4096 * 2];   // one quantised row (cols <= 4096, up to 2 bytes each)
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
  const float is = 1.0f / s;
  // the quantised row once into shared memory, then 16-byte stores of it to every destination
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int g = warp + 8 * i;
    if (g < ng) {
      if (PREC == VQ2_PREC_FP8) {
        qrow[g * 64 + lane] = (uint8_t)__nv_cvt_float_to_fp8(va[i] * s, __NV_SATFINITE, __NV_E4M3);
        qrow[g * 64 + 32 + lane] = (uint8_t)__nv_cvt_float_to_fp8(vb[i] * s, __NV_SATFINITE, __NV_E4M3);
      } else {
        ((__half*)qrow)[g * 64 + lane] = __float2half_rn(va[i] * s);
        ((__half*)qrow)[g * 64 + 32 + lane] = __float2half_rn(vb[i] * s);
      }
    }
  }
  __syncthreads();
  const int n16 = cols * elem / 16;             // cols is a multiple of 64: whole 16-byte words
  const int ndst = pslot ? k : 1;
  for (int jd = 0; jd < ndst; ++jd) {
    long dst = row;
    if (pslot) {
      dst = pslot[row * k + jd];
      if (dst < 0) continue;                    // pair owned by another device
    }
    uint4* orow_d = (uint4*)(out + dst * (size_t)cols * elem);
    if (threadIdx.x == 0) inv[dst] = is;
    for (int c = threadIdx.x; c < n16; c += blockDim.x) orow_d[c] = ((const uint4*)qrow)[c];
  }
}

// Warp-per-row variant for fp32 rows of at most 2048 columns (the intermediate rows of the down
// projection): one warp holds its whole row in registers (lane: elements lane and lane + 32 of
// every 64-group, all loads issued together), rotates every group with the shuffle FWHT, takes
// the row absmax with a warp reduction and writes the quantised row; same arithmetic and outputs
// as had_quant_rows_kernel. 8 rows per 256-thread CTA.
template <int PREC>
__global__ void __launch_bounds__(256) had_quant_rows_warp_kernel(const float* __restrict__ x,
                                                                  const uint8_t* __restrict__ valid, long rows,
                                                                  int cols, uint8_t* __restrict__ out,
                                                                  float* __restrict__ inv) {
  constexpr int NG = 32;                          // groups per row at most (2048 columns)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * 8 + warp;
  if (row >= rows) return;
  const int ng = cols / 64;
  const int elem = PREC == VQ2_PREC_FP8 ? 1 : 2;
  uint8_t* orow = out + row * (size_t)cols * elem;
  if (!valid[row]) {
    for (int c = lane; c < cols * elem / 4; c += 32) ((uint32_t*)orow)[c] = 0u;
    if (lane == 0) inv[row] = 0.f;
    return;
  }
  const float* xr = x + row * (size_t)cols;
  float va[NG], vb[NG];
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    va[g] = g < ng ? __ldcs(xr + g * 64 + lane) : 0.f;       // read once: streaming loads
    vb[g] = g < ng ? __ldcs(xr + g * 64 + 32 + lane) : 0.f;
  }
  float amax = 0.f;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    float a = va[g], b = vb[g];
    const float t = a + b;
    b = a - b;
    a = t;
#pragma unroll
    for (int len = 16; len >= 1; len >>= 1) {
      const float pa = __shfl_xor_sync(0xffffffffu, a, len), pb = __shfl_xor_sync(0xffffffffu, b, len);
      a = (lane & len) ? (pa - a) : (a + pa);
      b = (lane & len) ? (pb - b) : (b + pb);
    }
    va[g] = a * 0.125f;
    vb[g] = b * 0.125f;
    amax = fmaxf(amax, fmaxf(fabsf(va[g]), fabsf(vb[g])));
  }
  amax = warp_max(amax);
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
  if (lane == 0) inv[row] = 1.0f / s;
#pragma unroll
  for (int g = 0; g < NG; ++g) {
    if (g < ng) {
      if (PREC == VQ2_PREC_FP8) {
        orow[g * 64 + lane] = (uint8_t)__nv_cvt_float_to_fp8(va[g] * s, __NV_SATFINITE, __NV_E4M3);
        orow[g * 64 + 32 + lane] = (uint8_t)__nv_cvt_float_to_fp8(vb[g] * s, __NV_SATFINITE, __NV_E4M3);
      } else {
        ((__half*)orow)[g * 64 + lane] = __float2half_rn(va[g] * s);
        ((__half*)orow)[g * 64 + 32 + lane] = __float2half_rn(vb[g] * s);
      }
    }
  }
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
  size_t off_st, off_ss, off_val, off_be, off_counts, off_xs, off_invxs, off_inter, off_vb,
      off_invvb, off_chunks, off_nchunks, off_ranges, off_pslot, total;
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
  L.off_xs = o; o = up256(o + (size_t)L.Pmax * H * elem);
  L.off_invxs = o; o = up256(o + (size_t)L.Pmax * 4);
  L.off_inter = o; o = up256(o + (size_t)L.Pmax * I * 4);
  L.off_vb = o; o = up256(o + (size_t)L.Pmax * I * elem);
  L.off_invvb = o; o = up256(o + (size_t)L.Pmax * 4);
  L.off_chunks = o; o = up256(o + (size_t)L.nblk * 16);
  L.off_nchunks = o; o = up256(o + 4);
  L.off_ranges = o; o = up256(o + (size_t)E * 8);
  L.off_pslot = o; o = up256(o + (size_t)L.M * 4);
  L.total = o + 256;
  return L;
}

static bool g_pf_attr[64];
static int g_pf_pairs[64];   // resident CTA pairs of the GEMM kernels, per device

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
  uint8_t* xs = w + L.off_xs;
  float* invxs = (float*)(w + L.off_invxs);
  float* inter = (float*)(w + L.off_inter);
  uint8_t* vb = w + L.off_vb;
  float* invvb = (float*)(w + L.off_invvb);
  int4* chunks = (int4*)(w + L.off_chunks);
  int* nchunks = (int*)(w + L.off_nchunks);
  int2* ranges = (int2*)(w + L.off_ranges);
  int32_t* pslot = (int32_t*)(w + L.off_pslot);
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
  if (nsm < 2) return VQ2_ERR_CUDA;
  int rc = launch_align_ex(a->topk_ids, a->ids_dtype, a->N, a->topk, a->E, P2_BM, a->expert_base, 1, st, ss, val,
                           be, counts, st_, ranges, pslot);
  if (rc) return rc;
  if (cudaMemsetAsync(a->out, 0, (size_t)a->N * a->H * sizeof(float), st_) != cudaSuccess) return VQ2_ERR_CUDA;
  build_chunks_kernel<<<1, 1024, 0, st_>>>(ranges, a->E, chunks, nchunks);

  P2Args g = {};
  g.chunks = chunks; g.nchunks = nchunks;
  g.st = st; g.ss = ss; g.val = val; g.topk_w = a->topk_w; g.inter = inter; g.out = a->out;
  g.I = a->I; g.H = a->H; g.topk = a->topk;
  // Hadamard + per-token quantisation, each token row written to its slots (padding slots are
  // left as they are: their columns of the GEMMs are never combined into the output)
  if (prec == VQ2_PREC_FP8)
    had_quant_rows_kernel<VQ2_PREC_FP8><<<a->N, 256, 0, st_>>>(a->x, a->x_dtype, nullptr, a->H, xs, invxs, pslot, a->topk);
  else
    had_quant_rows_kernel<VQ2_PREC_F16><<<a->N, 256, 0, st_>>>(a->x, a->x_dtype, nullptr, a->H, xs, invxs, pslot, a->topk);
  const int elem = prec == VQ2_PREC_FP8 ? 1 : 2;
  CUtensorMap tm_x, tm_v, tm_l13, tm_l2;
  if (encode_2d(&tm_x, xs, (uint64_t)a->H * elem, L.Pmax, 128, P2_NSUB / 2, true) ||
      encode_2d(&tm_v, vb, (uint64_t)a->I * elem, L.Pmax, 128, P2_NSUB / 2, true) ||
      encode_2d(&tm_l13, a->w13_lo, a->H / 4, (uint64_t)a->E * 2 * a->I, 16, 64, false) ||
      encode_2d(&tm_l2, a->w2_lo, a->I / 4, (uint64_t)a->E * a->H, 16, 64, false))
    return VQ2_ERR_CUDA;
  // CTA pairs (clusters of 2), one CTA per SM: as many pairs as can be resident at once
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(nsm & ~1));
  cfg.blockDim = dim3(P2_THREADS);
  cfg.dynamicSmemBytes = P2_SMEM;
  cfg.stream = st_;
  cudaLaunchAttribute cattr[1];
  cattr[0].id = cudaLaunchAttributeClusterDimension;
  cattr[0].val.clusterDim.x = 2;
  cattr[0].val.clusterDim.y = 1;
  cattr[0].val.clusterDim.z = 1;
  cfg.attrs = cattr;
  cfg.numAttrs = 1;
  if (!g_pf_pairs[dev]) {
    int nc = 0;
    if (cudaOccupancyMaxActiveClusters(&nc, (void*)prefill_gemm_kernel<VQ2_PREC_FP8, true>, &cfg) != cudaSuccess || nc < 1)
      nc = nsm / 2;
    g_pf_pairs[dev] = std::min(nc, nsm / 2);
  }
  cfg.gridDim = dim3((unsigned)(2 * g_pf_pairs[dev]));
  // gate/up: row tiles of 128 gate + 128 up rows
  g.inv_slot = invxs; g.lo = a->w13_lo; g.hi = a->w13_hi; g.sc = a->w13_sc; g.cb = a->w13_cb;
  g.K = a->H; g.R = 2 * a->I; g.T = a->I / P2_ROWS;
  cudaError_t le = prec == VQ2_PREC_FP8 ? cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<VQ2_PREC_FP8, true>, g, tm_x, tm_l13)
                                        : cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<VQ2_PREC_F16, true>, g, tm_x, tm_l13);
  if (le != cudaSuccess) return VQ2_ERR_CUDA;
  // inter -> Hadamard -> quantised activation of the down projection
  if (a->I <= 2048) {
    const unsigned nb = (unsigned)((L.Pmax + 7) / 8);
    if (prec == VQ2_PREC_FP8)
      had_quant_rows_warp_kernel<VQ2_PREC_FP8><<<nb, 256, 0, st_>>>(inter, val, L.Pmax, a->I, vb, invvb);
    else
      had_quant_rows_warp_kernel<VQ2_PREC_F16><<<nb, 256, 0, st_>>>(inter, val, L.Pmax, a->I, vb, invvb);
  } else if (prec == VQ2_PREC_FP8) {
    had_quant_rows_kernel<VQ2_PREC_FP8><<<(unsigned)L.Pmax, 256, 0, st_>>>(inter, VQ2_DT_F32, val, a->I, vb, invvb,
                                                                            nullptr, 1);
  } else {
    had_quant_rows_kernel<VQ2_PREC_F16><<<(unsigned)L.Pmax, 256, 0, st_>>>(inter, VQ2_DT_F32, val, a->I, vb, invvb,
                                                                            nullptr, 1);
  }
  // down + combine: row tiles of 256 output rows
  g.inv_slot = invvb; g.lo = a->w2_lo; g.hi = a->w2_hi; g.sc = a->w2_sc; g.cb = a->w2_cb;
  g.K = a->I; g.R = a->H; g.T = a->H / (2 * P2_ROWS);
  le = prec == VQ2_PREC_FP8 ? cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<VQ2_PREC_FP8, false>, g, tm_v, tm_l2)
                            : cudaLaunchKernelEx(&cfg, prefill_gemm_kernel<VQ2_PREC_F16, false>, g, tm_v, tm_l2);
  if (le != cudaSuccess) return VQ2_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? VQ2_OK : VQ2_ERR_CUDA;
}
