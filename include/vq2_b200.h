/* vq2_b200 — C ABI of the B200 (sm_100a) vq2 routed-expert MoE path.
 *
 * A drop-in for the kernel layer of the vq2 vLLM plugin (iggerask/deepseek-v4-flash-2bit-gb10).
 * Plain pointers and sizes only; every pointer is DEVICE memory unless stated; the caller owns
 * all buffers (the library never allocates); every launch goes on the `stream` argument
 * (a cudaStream_t passed as void*; NULL = legacy default stream). Functions return 0 on success
 * or a VQ2_ERR_* code (see vq2_strerror); no exceptions cross the ABI and no kernel traps.
 *
 * Weight format (reference vq2_vllm/__init__.py:164-173), 10-bit index planes, 4-wide codebook,
 * group-64 scales and group-64 Hadamard incoherence folded into the activation:
 *   w13_lo [E,2I,H/4] u8   w13_hi [E,2I,H/16] u8   w13_sc [E,2I,H/64] f16   (rows 0..I-1 gate,
 *   w2_lo  [E,H,I/4]  u8   w2_hi  [E,H,I/16]  u8   w2_sc  [E,H,I/64]  f16    rows I..2I-1 up)
 *   w13_cb, w2_cb [1024,4] f16
 * Index of sub-vector s of a row: lo[s] | ((hi[s>>2] >> 2*(s&3)) & 3) << 8
 * (reference vq2_vllm/kernels/vq2_kernel.py:491-498, :534-535).
 */
#ifndef VQ2_B200_H
#define VQ2_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  VQ2_OK = 0,
  VQ2_ERR_NULL = 1,          /* a required pointer is NULL */
  VQ2_ERR_SHAPE = 2,         /* unsupported or inconsistent dimensions */
  VQ2_ERR_ALIGN = 3,         /* a pointer is not 16-byte aligned */
  VQ2_ERR_DTYPE = 4,         /* unknown dtype code */
  VQ2_ERR_WORKSPACE = 5,     /* workspace NULL or smaller than the *_workspace_size answer */
  VQ2_ERR_TOO_MANY_PAIRS = 6,/* decode path: N*topk above VQ2_DECODE_MAX_PAIRS */
  VQ2_ERR_CUDA = 7,          /* a CUDA runtime call failed (launch / attribute) */
  VQ2_ERR_TIMEOUT = 8,       /* a bounded device wait gave up (reported by vq2_device_status) */
  VQ2_ERR_NO_DEVICE = 9,     /* no sm_100 device is current */
  VQ2_ERR_NOALLOC_LIMIT = 10 /* vq2_decode_noalloc: the call needs more scratch than its fixed array */
};

enum { VQ2_DT_BF16 = 0, VQ2_DT_F16 = 1, VQ2_DT_F32 = 2 };   /* activation dtypes */
enum { VQ2_ID_I32 = 0, VQ2_ID_I64 = 1 };                      /* topk_ids dtypes  */
enum { VQ2_PREC_FP8 = 0, VQ2_PREC_F16 = 1 };                 /* prefill operand precision */

#define VQ2_DECODE_MAX_PAIRS 512

typedef struct vq2_moe_args {
  int N;            /* tokens */
  int H;            /* hidden size (multiple of 64, <= 4096) */
  int I;            /* expert intermediate size (multiple of 64, <= 4096) */
  int E;            /* routed experts held by this call (local experts under expert parallelism) */
  int topk;         /* experts per token */
  int x_dtype;      /* VQ2_DT_* */
  int ids_dtype;    /* VQ2_ID_* */
  int expert_base;  /* ids are global: local expert = id - expert_base; pairs whose local id falls
                       outside [0,E) are skipped (expert parallelism). 0 for a single device. */
  const void* x;         /* [N,H] */
  const void* topk_ids;  /* [N,topk] */
  const float* topk_w;   /* [N,topk] fp32 */
  const uint16_t* w13_cb; const uint8_t* w13_lo; const uint8_t* w13_hi; const uint16_t* w13_sc;
  const uint16_t* w2_cb;  const uint8_t* w2_lo;  const uint8_t* w2_hi;  const uint16_t* w2_sc;
  float* out;            /* [N,H] fp32, fully overwritten */
} vq2_moe_args;

/* Decode MoE (small token batches). Replaces vq2_kernel.vq2_moe_fused_10b
 * (reference vq2_vllm/kernels/vq2_kernel.py:569-594): out = sum_j w_nj * down_e(H·(silu(gate_e(Hx)) * up_e(Hx))).
 * Two kernels chained with programmatic dependent launch; no host sync, no allocation, safe to
 * capture in a CUDA graph. Requires N*topk <= VQ2_DECODE_MAX_PAIRS. */
size_t vq2_decode_workspace_size(int N, int topk, int H, int I);
int vq2_decode(const vq2_moe_args* a, void* workspace, size_t ws_bytes, void* stream);

/* Decode step from host buffers (no counterpart in the reference, whose callers hold device
 * tensors): for callers whose token rows, routing and result live in host memory. Queues on
 * `stream` the copies of h_x [N,H] (x_dtype), h_ids [N,topk] (ids_dtype) and h_w [N,topk] f32 into
 * the caller's device `stage`, the two decode kernels and the copy of out [N,H] f32 into h_out;
 * returns without waiting (synchronise the stream before reading h_out). Host buffers should be
 * page-locked for the copies to run asynchronously. In `a` only the dimensions, dtypes, E,
 * expert_base and the weight pointers are read; x, topk_ids, topk_w and out are taken from the
 * stage. workspace as for vq2_decode. */
size_t vq2_decode_host_stage_size(int N, int topk, int H, int x_dtype, int ids_dtype);
int vq2_decode_host(const vq2_moe_args* a, const void* h_x, const void* h_ids, const float* h_w, float* h_out,
                    void* stage, size_t stage_bytes, void* workspace, size_t ws_bytes, void* stream);

/* Pipelined host-buffer decode step (no counterpart in the reference): h_in holds the step's
 * inputs packed as x | ids | w at the offsets vq2_decode_host_offsets gives (each part 256-byte
 * aligned; in_bytes in total); d_in is device memory of in_bytes (256-byte aligned), d_out the
 * device result [N,H] f32. The upload runs on in_stream and records ev_in; `stream` waits for it
 * and runs the decode kernels, then records ev_done; out_stream waits for that, downloads the
 * result into h_out and records ev_out. Events (cudaEvent_t as void*, one set per staging slot,
 * recorded at least once before the first use) and streams are the caller's; a slot's previous
 * ev_done / ev_out order its new upload and kernels after that step's kernels and download. With
 * separate upload and download streams the copies of neighbouring steps overlap the kernels.
 * x, topk_ids, topk_w and out in `a` are ignored. Host buffers should be page-locked. */
void vq2_decode_host_offsets(int N, int topk, int H, int x_dtype, int ids_dtype, size_t* off_ids, size_t* off_w,
                             size_t* in_bytes);
int vq2_decode_host_async(const vq2_moe_args* a, const void* h_in, float* h_out, void* d_in, float* d_out,
                          void* workspace, size_t ws_bytes, void* stream, void* in_stream, void* out_stream,
                          void* ev_in, void* ev_done, void* ev_out);

/* Allocation-free decode: no counterpart in the reference. For callers that cannot allocate
 * device memory when they call (a memory pool that forbids new allocations, a driver callback, a
 * host runtime without a CUDA allocator): same result as vq2_decode, but the gate/up scratch is a
 * fixed array inside the library (VQ2_NOALLOC_SCRATCH_BYTES, reserved on every GPU that loads the
 * library until the process exits) instead of a caller workspace. The call allocates nothing.
 * Limit: N*topk*ceil(H/2048)*2*I*4 bytes <= VQ2_NOALLOC_SCRATCH_BYTES, else VQ2_ERR_NOALLOC_LIMIT
 * (2 MiB: 64 token-expert pairs at H=4096, I=2048, i.e. 8 decode tokens at top-8).
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture. All calls share the array:
 * calls that overlap on the GPU (other streams, other threads) race and corrupt each other. */
#define VQ2_NOALLOC_SCRATCH_BYTES (2u << 20)
int vq2_decode_noalloc(const vq2_moe_args* a, void* stream);

/* Prefill MoE (grouped GEMM on tcgen05 tensor cores). Replaces ds4_vq2_cuda.vq2_moe_grouped_wmma
 * (reference vq2_vllm/kernels/ds4_vq2_cuda.py:72-111). precision = VQ2_PREC_FP8 follows the
 * reference's fp8 e4m3 algorithm; VQ2_PREC_F16 runs fp16 operands (activations scaled by a power of two
 * into fp16 range, fp32 accumulation) and meets 3e-2 against the fp32 dequant reference. */
size_t vq2_prefill_workspace_size(int N, int topk, int E, int H, int I, int precision);
int vq2_prefill(const vq2_moe_args* a, int precision, void* workspace, size_t ws_bytes, void* stream);

/* moe_align: stable sort of (token, slot) pairs by expert, padded to BM per expert. Replaces
 * moe_align.moe_align / _moe_align_torch (reference vq2_vllm/kernels/moe_align.py:50-86),
 * bit-exact with the latter. Pmax = M + min(M,E)*BM, nblk = Pmax/BM (M = N*k). Outputs:
 * sorted_tok i32[Pmax], sorted_slot i32[Pmax], valid u8[Pmax], block_e i32[nblk]. Ids outside
 * [0,E) are clamped, as the reference's prefill wrapper does (ds4_vq2_cuda.py:82-85). */
size_t vq2_align_workspace_size(int N, int k, int E);
int vq2_align(const void* topk_ids, int ids_dtype, int N, int k, int E, int BM,
              int32_t* sorted_tok, int32_t* sorted_slot, uint8_t* valid, int32_t* block_e,
              void* workspace, size_t ws_bytes, void* stream);

/* Per-row absmax fp8 e4m3 quantisation: s = 448/max(amax,1e-6); out = e4m3(x*s); inv = 1/s.
 * Replaces ds4_vq2_cuda.quant_fp8_rows (reference vq2_vllm/kernels/ds4_vq2_cuda.py:8-32). */
int vq2_quant_fp8_rows(const float* x, int rows, int cols, uint8_t* out, float* inv, void* stream);

/* Group-64 Hadamard of each row, X @ H per group (H Sylvester, 1/8 normalised). in/out dtype
 * VQ2_DT_*; cols a multiple of 64. Replaces vq2_kernel.had_act_batch
 * (reference vq2_vllm/kernels/vq2_kernel.py:188-195). */
int vq2_hadamard_rows(const void* x, int in_dtype, void* y, int out_dtype, long rows, int cols, void* stream);

/* ---- expert-parallel token exchange over NVLink peer memory (no counterpart in the reference,
   which runs on one device). One exchange region per rank, allocated by vq2_ep_alloc (zeroed) and
   shared through CUDA IPC handles; regions are laid out identically on every rank:
     X    [world][N][row_x]   token rows as pushed by each source rank (bytes, 16-byte multiple)
     IDS  [world][N][k] i32   their expert ids
     WT   [world][N][k] f32   their routing weights
     COMB [world][N][H] f32   partial outputs pushed back by each rank, for this rank's tokens
     DFLAG[world][VQ2_EP_CTAS] u32, CFLAG[world][VQ2_EP_CTAS] u32   per-(source, slice) step flags
     EPOCH u32   this rank's step
     COUNT u32[2]   completion counter of the fused step's down kernel (vq2_ep_decode)
   `peers` is a device array [world][6] of u64 addresses (X, IDS, WT, COMB, DFLAG, CFLAG) of every
   rank's region, this rank's included. Every rank calls dispatch / combine once per step with the
   same N. Waits are bounded: a peer that never arrives makes vq2_device_status report
   VQ2_ERR_TIMEOUT, and the call returns with the data it has. */
#define VQ2_EP_CTAS 8   /* at most this many slices (CTAs, flags) per destination: one per 32 KB */
int vq2_ep_alloc(size_t bytes, void** dev_ptr_out);
int vq2_ep_free(void* dev_ptr);
int vq2_ipc_get_handle(const void* dev_ptr, void* handle_out /* 64 bytes */);
int vq2_ipc_open(const void* handle /* 64 bytes */, void** dev_ptr_out);
int vq2_ipc_close(void* dev_ptr);
/* Push this rank's N rows (x: N x row_x bytes; ids N x k of VQ2_ID_I32 / VQ2_ID_I64, stored as
   i32; w f32 N x k) into slot `rank` of every rank's X/IDS/WT, signal, and wait until every rank's
   rows have arrived here. */
int vq2_ep_dispatch(const void* x, const void* ids, int ids_dtype, const float* w, int N, int row_x, int k,
                    const uint64_t* peers, int world, int rank, void* my_region, size_t off_dflag,
                    size_t off_epoch, void* stream);
/* part: f32 [world*N][H], rows [d*N, (d+1)*N) belong to rank d's tokens. Push them into slot
   `rank` of rank d's COMB, signal, wait for every rank's rows, and write out[n][h] = sum over
   source ranks of COMB[src][n][h] (f32 [N][H]). */
int vq2_ep_combine(const float* part, int N, int H, const uint64_t* peers, int world, int rank,
                   void* my_region, size_t off_comb, size_t off_cflag, size_t off_epoch, float* out,
                   void* stream);

/* Byte offsets of the region's fields (every one a multiple of 16; the same on every rank). */
typedef struct vq2_ep_layout {
  size_t off_x, off_ids, off_w, off_comb, off_dflag, off_cflag, off_epoch, off_count;
} vq2_ep_layout;
/* One expert-parallel decode step with the exchange fused into the decode kernels (replaces
   dispatch + vq2_decode on the gathered rows + combine; the reference's decode call
   vq2_vllm/kernels/vq2_kernel.py:569-594 runs on one device). `a` is this rank's call: x, topk_ids,
   topk_w of its N tokens (global expert ids), `out` f32 [N][H], and this rank's experts (a->E
   experts from a->expert_base). A small push kernel stores the rows into every rank's region;
   the gate/up kernel waits for every rank's; both decode kernels run over the world*N gathered
   tokens; the down kernel adds each result into its owner's COMB rows with fp32 atomics over
   NVLink (so the sum order over ranks is not fixed), and its last CTA waits for every rank's
   completion flag, writes `out` and re-zeroes COMB. Every rank calls it once per step with the
   same N; world*N*topk <= VQ2_DECODE_MAX_PAIRS. Three launches, no host synchronisation. Do not mix with dispatch / combine on one region. */
size_t vq2_ep_decode_workspace_size(int world, int N, int topk, int H, int I);
int vq2_ep_decode(const vq2_moe_args* a, const uint64_t* peers, int world, int rank, void* my_region,
                  const vq2_ep_layout* layout, void* ws, size_t ws_bytes, void* stream);

/* ---- router (upstream of the MoE method): topk_w, topk_ids = top-k(softmax(x . W_r)) per token,
   weights = the selected probabilities (not renormalised); ids by probability descending, lower
   index first on ties. x: N x H of x_dtype; w_r: bf16 [H][E] (row-major, E contiguous); N <= 64,
   H % 64 == 0, E <= 1024, k <= min(E, 64). fp32 logits summed in a fixed order (deterministic). */
size_t vq2_router_workspace_size(int N, int H, int E);
int vq2_router_topk(const void* x, int x_dtype, const void* w_r, int N, int H, int E, int k,
                    int32_t* topk_ids, float* topk_w, void* workspace, size_t ws_bytes, void* stream);

/* ---- VQ packer (offline quantisation into the format above; not on the serving path). Replaces
   the k-means packer vq2_kernel.pack_vq2 (reference vq2_vllm/kernels/vq2_kernel.py:37-72). W is
   [rows][D] of VQ2_DT_* (columns zero-padded to ng = ceil(D/64) groups); sub-vectors are numbered
   flat over rows x groups x 16 (sub-vector v: group v>>4, columns 4*(v&15)..+3 of the rotated
   group). Rotation is the group Hadamard (fp32 butterfly), scale s = max(|group|, 1e-8), values
   normalised by s; distances ((d0^2+d1^2)+d2^2)+d3^2 with each operation rounded separately, lowest
   index on ties; k <= 1024. */
/* out f32 [n][4] (16-byte aligned): the normalised sub-vectors vec_idx[0..n). An index outside
   [0, rows*ng*16) is skipped (its output row is left as it was) and vq2_device_status reports
   VQ2_ERR_SHAPE. */
int vq2_pack_gather(const void* W, int w_dtype, long long rows, int D, const long long* vec_idx, long long n,
                    float* out, void* stream);
/* `iters` Lloyd iterations over samp f32 [n][4] starting from C f32 [k][4] (updated in place): each
   centroid with members becomes their mean (members summed as int64 fixed point, value x 2^40
   rounded to nearest even; mean = (double)sum * 2^-40 / count rounded to f32); empty ones stay.
   samp values must be at most 1 in magnitude (the normalised sub-vectors vq2_pack_gather writes)
   and n <= 2^23 (VQ2_ERR_SHAPE above), so the int64 sums cannot overflow. */
size_t vq2_kmeans_workspace_size(int k);
int vq2_kmeans(const float* samp, long long n, float* C, int k, int iters, void* workspace, size_t ws_bytes,
               void* stream);
/* Nearest centroid of every sub-vector of W. Outputs (each optional except scale):
   lo u8 [rows*ng*16] and hi u8 [rows*ng*4] (the 10-bit planes, both or neither, lo 4-byte aligned),
   idx i16 [rows*ng*16] (8-byte aligned), scale f32 [rows*ng], dq f32 [rows][D] = (C[id] * s) @ H64. */
int vq2_pack_assign(const void* W, int w_dtype, long long rows, int D, const float* C, int k, uint8_t* lo,
                    uint8_t* hi, int16_t* idx, float* scale, float* dq, void* stream);

/* ---- shared expert of the decode step (no counterpart in the reference plugin, whose `apply`
   leaves it to vLLM): out[n] (+)= W2 . (silu(Wg . x[n]) * (Wu . x[n])), dense bf16 weights
   w13 = [Wg; Wu] [2*Is][H] and w2 [H][Is] (row-major, 16-byte aligned), fp32 accumulation and
   fp32 intermediate. out f32 [N][H]: overwritten, or added to with accumulate = 1. N <= 8,
   H and Is multiples of 256, N*H*4 and N*Is*4 <= 200 KB. Two launches chained by programmatic
   dependent launch; the first waits for the stream's previous work, so `out` may be the routed
   experts' output of the same stream. */
size_t vq2_shared_expert_workspace_size(int N, int Is);
int vq2_shared_expert(const void* x, int x_dtype, const void* w13, const void* w2, int N, int H, int Is, float* out,
                      int accumulate, void* workspace, size_t ws_bytes, void* stream);

/* Routed decode plus the shared expert in one call: out = routed MoE (as vq2_decode) + the shared
   expert (as vq2_shared_expert with sw13 / sw2 / Is) for the same x, fp32 [N][H] (N <= 8 for the
   shared part). The routed kernels run on (SMs - shared_sms) SMs and the shared expert's kernels
   concurrently on shared_sms SMs (<= 0: VQ2_SHARED_SMS_DEFAULT) on a second stream this library
   creates per device, forked from and joined into `stream` with events (capturable in a CUDA
   graph once the first call on the device, which creates that stream and its events, has run
   outside capture); both add into `out` with fp32 atomics after one zeroing, so the sum order is not fixed.
   Workspace: vq2_decode_with_shared_workspace_size. No reference counterpart as one call: vLLM
   runs the shared expert beside the MoE method (reference vq2_vllm/__init__.py:197-198). */
#define VQ2_SHARED_SMS_DEFAULT 56   /* best of a 12..110 sweep at config 1, batch 1 */
size_t vq2_decode_with_shared_workspace_size(int N, int topk, int H, int I, int Is);
int vq2_decode_with_shared(const vq2_moe_args* a, const void* sw13, const void* sw2, int Is, int shared_sms,
                           void* ws, size_t ws_bytes, void* stream);

/* Error word written by bounded device waits and device-side range checks (0 = none);
   reset = 1 clears it. Synchronises the device. */
int vq2_device_status(int reset);
const char* vq2_strerror(int code);
int vq2_version(void);

#ifdef __cplusplus
}
#endif
#endif /* VQ2_B200_H */
