// Shared device helpers for the vq2 sm_100a kernels: bounded mbarrier waits, 1-D bulk async
// copies (TMA engine), PDL control, warp reductions, the 64-point Walsh-Hadamard transform and
// the in-CTA (token, slot) -> expert grouping used by the decode kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include "../../include/vq2_b200.h"

#define VQ2_WAIT_LIMIT (1u << 22)   // try_wait polls before a wait gives up (well under a second)

namespace vq2 {

// Error word set by a wait that gave up; read by vq2_device_status(). The library is built as
// one translation unit (vq2_lib.cu), so this is its only definition.
__device__ int g_status = 0;

__device__ __forceinline__ void set_status(int code) { atomicCAS(&g_status, 0, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---------------------------------------------------------------- explicit shared-window access
// 32-bit shared-window addresses keep these on the shared-memory path (no generic-address
// resolution). lds64: data-dependent gathers from tables written before a barrier (free to be
// scheduled by the compiler). The volatile forms read ring slots / write tiles whose order against
// mbarrier waits, fences and arrivals matters.
__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds128_v(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint2 lds64_v(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds32_v(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds16_v(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds8_v(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void sts128_v(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait: returns false (and records VQ2_ERR_TIMEOUT) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < VQ2_WAIT_LIMIT; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  set_status(VQ2_ERR_TIMEOUT);
  return false;
}

// ---------------------------------------------------------------- bulk async copy (1-D TMA)
// global -> shared, completion counted on `bar` in bytes. src, dst 16-B aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Streaming variant: the lines are marked evict-first in L2 (`policy` from l2_evict_first()), so a
// once-read weight stream does not push code, activations and partials out of L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy) : "memory");
}

// ---------------------------------------------------------------- expert-parallel exchange flags
// Shared by the stand-alone exchange kernels and the decode kernels' fused exchange.
// Ordering: every thread of the CTA stores its share of the data, the CTA barrier orders those
// stores before the signalling thread's next operations, and the signalling thread's release
// store at system scope (a fence.acq_rel.sys plus the store) makes everything ordered before it
// visible to a peer thread whose acquire load reads the flag (causality is transitive through
// the barrier). No separate sequentially-consistent fence is needed (measured: it cost ~2 us
// per handshake).
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until the flag has reached step `ep` (wrap-safe comparison).
__device__ __forceinline__ bool ep_wait_flag(const unsigned* f, unsigned ep) {
  for (uint32_t i = 0; i < VQ2_WAIT_LIMIT; ++i) {
    if ((int)(ld_acquire_sys(f) - ep) >= 0) return true;
    __nanosleep(32);
  }
  set_status(VQ2_ERR_TIMEOUT);
  return false;
}

enum { EP_X = 0, EP_IDS = 1, EP_WT = 2, EP_COMB = 3, EP_DFLAG = 4, EP_CFLAG = 5, EP_FIELDS = 6 };

// Slice [c * chunk, (c + 1) * chunk) of `bytes`, chunk a multiple of `align` (16 or 4).
__device__ __forceinline__ void ep_slice(size_t bytes, int c, int C, size_t align, size_t& b, size_t& e) {
  const size_t chunk = ((bytes + C - 1) / C + align - 1) / align * align;
  b = min(bytes, (size_t)c * chunk);
  e = min(bytes, b + chunk);
}

// Slices per destination: about one per 32 KB pushed, 1..VQ2_EP_CTAS. Every rank derives the same
// count from the same N, so senders and receivers agree on the number of flags.
__host__ __device__ __forceinline__ int ep_slices(size_t bytes_per_dest) {
  const size_t s = (bytes_per_dest + 32767) / 32768;
  return s < 1 ? 1 : (s > VQ2_EP_CTAS ? VQ2_EP_CTAS : (int)s);
}

// ---------------------------------------------------------------- programmatic dependent launch
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// In-register 64-point Walsh-Hadamard transform in natural (Sylvester) order, unnormalised:
// y_j = sum_i x_i (-1)^popcount(i&j), i.e. x @ (8 H64) with H64 the reference's normalised
// Sylvester matrix (vq2_vllm/kernels/vq2_kernel.py:18-22).
__device__ __forceinline__ void fwht64(float* v) {
#pragma unroll
  for (int len = 1; len < 64; len <<= 1) {
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      if ((i & len) == 0) {
        float a = v[i], b = v[i + len];
        v[i] = a + b;
        v[i + len] = a - b;
      }
    }
  }
}

// Power-of-two scale that maps a max magnitude `amax` to at most 2^14, so fp16 storage of
// activations cannot overflow (returned as (scale, inverse)). amax == 0 -> 1.
__device__ __forceinline__ float2 f16_range_scale(float amax) {
  if (!(amax > 0.f)) return make_float2(1.f, 1.f);
  int ex;
  frexpf(amax, &ex);                 // amax in [2^(ex-1), 2^ex)
  int s = 14 - ex;                   // amax * 2^s < 2^14
  s = max(-60, min(60, s));
  return make_float2(ldexpf(1.f, s), ldexpf(1.f, -s));
}

// The four 10-bit indices of one lo word (4 index low bytes) and its hi byte hb (four 2-bit
// fields, sub-vector j in bits 2j..2j+1), as two words with two 16-bit ids each:
// ids02 = id0 | id2 << 16, ids13 = id1 | id3 << 16. Byte permutes place the low bytes; a multiply
// spreads hb into both halves so one masked OR adds the two hi bits.
__device__ __forceinline__ void unpack_ids4(uint32_t lo_word, uint32_t hb, uint32_t& ids02, uint32_t& ids13) {
  const uint32_t e02 = __byte_perm(lo_word, 0u, 0x4240);   // [b0, 0, b2, 0]
  const uint32_t e13 = __byte_perm(lo_word, 0u, 0x4341);   // [b1, 0, b3, 0]
  ids02 = e02 | ((hb * 0x00100100u) & 0x03000300u);         // hb bits 0-1 -> 8-9, bits 4-5 -> 24-25
  ids13 = e13 | ((hb * 0x00040040u) & 0x03000300u);         // hb bits 2-3 -> 8-9, bits 6-7 -> 24-25
}

// The same four ids, each from one byte permute: ids_hi_pairs() spreads the hi byte (8 bits, two
// per id) into two words whose other bytes are zero — h02 = [h0, 0, h2, 0], h13 = [0, h1, 0, h3] —
// and id_of<j>() puts id j's low byte (from the lo word) and its high bits side by side.
__device__ __forceinline__ void ids_hi_pairs(uint32_t hb, uint32_t& h02, uint32_t& h13) {
  h02 = (hb * 0x1001u) & 0x00030003u;    // hb bits 0-1 -> byte 0, bits 4-5 -> byte 2
  h13 = (hb * 0x40040u) & 0x03000300u;   // hb bits 2-3 -> byte 1, bits 6-7 -> byte 3
}
template <int J>
__device__ __forceinline__ uint32_t id_of(uint32_t lo_word, uint32_t h02, uint32_t h13) {
  return __byte_perm(lo_word, (J & 1) ? h13 : h02, J == 0 ? 0x5540 : J == 1 ? 0x4451 : J == 2 ? 0x5562 : 0x4473);
}

// Streaming-multiprocessor count of the current device, looked up once per device (grids of the
// grid-stride kernels are sized from it). Returns 0 if the query fails.
inline int device_sm_count() {
  static int counts[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!counts[dev] && cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    counts[dev] = 0;
  return counts[dev];
}

// Packed fp32 multiply of two pairs (Blackwell mul.rn.f32x2: each half rounded on its own).
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  unsigned long long d, x, y;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b.x), "f"(b.y));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(x), "l"(y));
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(d));
  return r;
}

__device__ __forceinline__ int load_id(const void* ids, int ids_dtype, int m) {
  return ids_dtype == VQ2_ID_I64 ? (int)((const long long*)ids)[m] : ((const int*)ids)[m];
}

__device__ __forceinline__ float load_act(const void* x, int dt, size_t i) {
  if (dt == VQ2_DT_BF16) return __bfloat162float(((const __nv_bfloat16*)x)[i]);
  if (dt == VQ2_DT_F16) return __half2float(((const __half*)x)[i]);
  return ((const float*)x)[i];
}

}  // namespace vq2
