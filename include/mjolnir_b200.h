/*
 * mjolnir_b200 -- C ABI of the B200 (sm_100a) decode-attention hot path.
 *
 * Three device operations behind plain pointers, sizes and a cudaStream_t
 * passed as void*. No torch types, no allocation inside any call (the caller
 * owns every buffer, including the split-KV scratch), every call returns an
 * int status (MJ_OK = 0) and never aborts the process.
 *
 *   mj_cache_write  quantize-on-write of new K/V rows into the paged cache
 *                   (fp8-e4m3, or e2m3 packed 4 codes per 3 bytes)
 *   mj_decode       paged split-KV decode attention over that cache
 *   mj_combine      log-sum-exp merge of the split-KV partials
 *
 * Reference interfaces these replace (GoBrrr-ai/mjolnir, src/mjolnir/mjolnir/):
 *   mj_cache_write  kvfp6.py:218-254 `write_kv` (e2m3) and the fp8 write
 *                   `MjolnirImpl.do_kv_cache_update` -> vLLM
 *                   `reshape_and_cache_flash` (backend.py:474-483)
 *   mj_decode       arch/thor/runner.py:374-407 `T5DecodeRunner._launch`, the
 *                   compiled `decode` kernel (arch/thor/decode.py:243-1471,
 *                   launched by arch/thor/call.py:481-529)
 *   mj_combine      the `reduction` kernel (arch/thor/decode.py:1473-1541,
 *                   launched by arch/thor/call.py:536-560)
 *
 * Layout conventions
 *   Q / O        (tokens, h_q, head_size), token = seq * q_len + qi, head dim
 *                contiguous; token and head strides in ELEMENTS.
 *   K / V cache  logical views (num_pages, page_size, h_k, row_bytes) with the
 *                row (head_size elements, or head_size*3/4 packed e2m3 bytes)
 *                contiguous; page / row / head strides in BYTES (any physical
 *                layout: vLLM's (B, H, N, 2*row), FlashInfer NHD/HND, ...).
 *   block_table  int32 (>= num_seqs, block_table_stride); token t of sequence s
 *                lives in page block_table[s * stride + t / page_size].
 *   seq_lens     int32 (num_seqs,), INCLUDING the step's q_len new tokens.
 *   work         int32 (num_work, 4): (seq, tile_begin, tile_end, split) in
 *                128-row KV tiles; tile_begin == tile_end is an empty item.
 *   n_splits     int32 (num_seqs,): number of work items of each sequence.
 */
#ifndef MJOLNIR_B200_H
#define MJOLNIR_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MJ_ABI_VERSION 4

/* status codes */
#define MJ_OK 0
#define MJ_ERR_INVALID 1     /* an argument failed validation (see mj_last_error) */
#define MJ_ERR_UNSUPPORTED 2 /* a shape / format / alignment this build does not run */
#define MJ_ERR_CUDA 3        /* a CUDA runtime call failed (see mj_last_error) */
#define MJ_ERR_DEVICE 4      /* a kernel flagged a bad index in the device status word */

/* device status word codes (written by kernels into args->status, if given) */
#define MJ_DEV_OK 0
#define MJ_DEV_BAD_PAGE 1    /* block-table entry or slot page outside [0, num_pages) */
#define MJ_DEV_BAD_SPLIT 2   /* work item split >= max_splits or seq >= part_seqs */
#define MJ_DEV_TIMEOUT 3     /* a bounded wait in a pipelined kernel gave up */

/* KV formats. e2m3 / e3m2: 6-bit codes (sign | exponent | mantissa, biases
 * 1 / 3, maxima 7.5 / 28, no inf or NaN) packed 4 per 3 bytes little-endian;
 * e2m1: 4-bit codes (bias 1, max 6) packed 2 per byte, low nibble first
 * (arch/thor/decode.py:108-115, quant.py:14-65). nvfp4: e2m1 codes as e2m1
 * plus one e4m3 scale byte per 16 elements of a row in a separate scale
 * tensor (logical (num_pages, page_size, h_k, head_size / 16) bytes) and a
 * global fp32 scale gs; the value multiplied is e4m3(code * scale * 2^-3)
 * with descale gs * 2^3 (quant.py:68-84, arch/thor/decode.py:980-1030).
 * The vLLM path serves e4m3 and e2m3; the others are the reference
 * harness's formats. */
#define MJ_KV_FP8_E4M3 0
#define MJ_KV_E2M3 1
#define MJ_KV_E3M2 2
#define MJ_KV_E2M1 3
#define MJ_KV_NVFP4 4

/* element types of Q / O / new K,V rows */
#define MJ_DT_BF16 0
#define MJ_DT_FP16 1
#define MJ_DT_FP32 2

/* decode kernels: AUTO picks the tensor-core kernel when it can run the
 * arguments (head_size 128 or 256, page 16..128, TMA-aligned KV views), else the
 * CUDA-core kernel; TC demands the former. */
#define MJ_KERNEL_AUTO 0
#define MJ_KERNEL_SIMT 1
#define MJ_KERNEL_TC 2

/* scale / descale modes */
#define MJ_SCALE_TENSOR 0   /* one fp32 */
#define MJ_SCALE_HEAD 1     /* (h_k,) fp32 */
#define MJ_SCALE_CHANNEL 2  /* (h_k, head_size) fp32 -- cache write only */
#define MJ_SCALE_SEQ_HEAD 3 /* (num_seqs, h_k) fp32 -- decode descales only */

/* Last error message of the calling thread ("" when none). */
const char* mj_last_error(void);
/* MJ_ABI_VERSION of the loaded library. */
int mj_abi_version(void);
/* Bytes of one K (or V) row: head_size (fp8), head_size*3/4 (e2m3, e3m2) or head_size/2 (e2m1, nvfp4 codes); -1 if invalid. */
int mj_row_bytes(int head_size, int kv_format);

/* ------------------------------------------------------------------------ */
/* Quantize-on-write (reshape_and_cache).                                   */
/* Replaces kvfp6.py:218-254 write_kv and the fp8 reshape_and_cache_flash    */
/* call of backend.py:474-483. Token t with slot_mapping[t] >= 0 is written  */
/* to page slot / page_size, row slot % page_size; slot < 0 is skipped.      */
/* e2m3: x / scale in fp32 (IEEE division), round to nearest with ties to   */
/* the smaller magnitude, saturate at 7.5, no -0; codes packed little-endian */
/* (c0 | c1<<6 | c2<<12 | c3<<18 -> 3 bytes) -- quant.py:34-65.              */
/* fp8: x / scale in fp32, round to nearest even, saturate at +-448.         */
/* nvfp4 (quant.py:68-84 with a given global scale gs = k_scale / v_scale,  */
/* per tensor or per KV head): per group of 16 elements the scale byte      */
/* e4m3(min(amax / 6 / gs, 448)), then each code e2m1(x / (scale * gs)),    */
/* 0 where that product is 0; head_size a multiple of 128.                  */
typedef struct mj_cache_write_args {
  const void* key;              /* (num_tokens, h_k, head_size), head dim contiguous */
  const void* value;
  int src_dtype;                /* MJ_DT_BF16 | MJ_DT_FP16 | MJ_DT_FP32 */
  int64_t num_tokens;
  int h_k;
  int head_size;                /* multiple of 16 */
  int64_t key_stride_tok, key_stride_head;     /* elements */
  int64_t value_stride_tok, value_stride_head; /* elements */
  void* k_cache;                /* logical (num_pages, page_size, h_k, row_bytes) */
  void* v_cache;
  int64_t k_stride_page, k_stride_row, k_stride_head; /* bytes */
  int64_t v_stride_page, v_stride_row, v_stride_head; /* bytes */
  int64_t num_pages;
  int page_size;
  int kv_format;                /* MJ_KV_* */
  const int64_t* slot_mapping;  /* (num_tokens,) */
  const float* k_scale;         /* per k_scale_mode */
  int k_scale_mode;             /* MJ_SCALE_TENSOR | _HEAD | _CHANNEL */
  const float* v_scale;
  int v_scale_mode;
  int32_t* status;              /* optional device status word (MJ_DEV_*) */
  /* nvfp4 only: the group scale tensors, logical (num_pages, page_size, h_k, head_size / 16) bytes */
  void* k_scales;
  void* v_scales;
  int64_t ks_stride_page, ks_stride_row, ks_stride_head; /* bytes */
  int64_t vs_stride_page, vs_stride_row, vs_stride_head; /* bytes */
} mj_cache_write_args;

int mj_cache_write(const mj_cache_write_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Paged split-KV decode attention.                                          */
/* Query row n = qi * h_r + r of KV head h (h_r = h_q / h_k) reads token     */
/* seq * q_len + qi, q head h * h_r + r. With causal != 0, query token qi of */
/* a sequence of length L sees keys 0 .. L - q_len + qi, otherwise all L.    */
/* score = (q * q_mul) . k_code * softmax_scale * k_descale;                 */
/* O = softmax(score) . v_code * v_descale * o_mul. A row that sees no key   */
/* gets O = 0 and LSE = -inf.                                                 */
/* A work item whose sequence has n_splits == 1 writes the final O (and LSE);*/
/* otherwise it writes its chunk-normalized partial into o_part / lse_part   */
/* at [split][seq][h][n], merged by mj_combine (or by mj_decode itself when  */
/* with_combine != 0). No allocation: safe inside CUDA-graph capture.        */
typedef struct mj_decode_args {
  int num_seqs, q_len, h_q, h_k, head_size, page_size, kv_format;
  const void* q; int q_dtype; int64_t q_stride_tok, q_stride_head;  /* elements */
  void* o; int o_dtype; int64_t o_stride_tok, o_stride_head;        /* elements */
  const void* k_cache; const void* v_cache;
  int64_t k_stride_page, k_stride_row, k_stride_head;               /* bytes */
  int64_t v_stride_page, v_stride_row, v_stride_head;               /* bytes */
  int64_t num_pages;
  const int32_t* block_table; int64_t block_table_stride;
  const int32_t* seq_lens;
  const int32_t* work; int num_work;
  const int32_t* n_splits; int max_splits;
  float* o_part;    /* scratch (max_splits, part_seqs, h_k, n_q, head_size) fp32 */
  float* lse_part;  /* scratch (max_splits, part_seqs, h_k, n_q) fp32 */
  int part_seqs;    /* >= num_seqs when any sequence splits */
  float* lse;       /* optional (num_seqs * q_len, h_q) natural-log LSE */
  const float* k_descale; int k_descale_mode; /* MJ_SCALE_TENSOR | _HEAD | _SEQ_HEAD */
  const float* v_descale; int v_descale_mode;
  const float* q_mul;  /* optional (h_q, head_size): Q *= q_mul (e2m3 K channel scales) */
  const float* o_mul;  /* optional (h_q, head_size): O *= o_mul (e2m3 V channel scales) */
  float softmax_scale;
  int causal;
  int with_combine;    /* also run mj_combine after the decode */
  int kernel;          /* MJ_KERNEL_AUTO, MJ_KERNEL_SIMT or MJ_KERNEL_TC */
  int32_t* status;     /* optional device status word (MJ_DEV_*) */
  /* Optional (num_seqs * h_k * 64) int32 counters, zero before the first
   * call; the kernel leaves them zero again -- except after a device error
   * (a non-zero status word), when jobs may have stopped before counting
   * in: zero them again before the next call. With them, the tensor-core
   * kernel merges the split partials itself: the last job of each (sequence,
   * KV head, row group) to finish merges them and writes the final O / LSE,
   * so no mj_combine launch is needed (mj_decode skips it). Applies to the
   * variants of up to 16 query rows per KV head with max_splits <= 16; the
   * others, and the CUDA-core kernel, ignore the counters. Replaces the reference's planned last-CTA merge
   * (arch/thor/decode.py:1417-1469, plan.py:122-129). */
  int32_t* merge_counters;
  /* nvfp4 only: the group scale tensors, logical (num_pages, page_size, h_k,
   * head_size / 16) bytes, rows 8-byte aligned for the tensor-core kernel;
   * k_descale / v_descale carry gs * 2^3 (arch/thor/call.py:138-139, :343-356) */
  const void* k_scales;
  const void* v_scales;
  int64_t ks_stride_page, ks_stride_row, ks_stride_head; /* bytes */
  int64_t vs_stride_page, vs_stride_row, vs_stride_head; /* bytes */
  /* Test hook for the kernel's abort path; 0 in normal use. Every wait
   * inside the tensor-core kernel's pipeline is bounded (0.5 s; a tile takes
   * microseconds) and a wait that runs out sets MJ_DEV_TIMEOUT in the status
   * word; the kernel then stops, lets its copies and MMAs in flight finish,
   * frees its tensor memory and returns, leaving the context usable (the
   * reference's pipeline waits are unbounded). When non-zero, the MMA issuer
   * of every CTA first waits this many ns on a phase that nothing completes,
   * so that path runs on a normal launch. */
  uint64_t abort_probe_ns;
} mj_decode_args;

int mj_decode(const mj_decode_args* args, void* stream);

/* The kernel mj_decode would launch for these arguments: MJ_KERNEL_SIMT or
 * MJ_KERNEL_TC (a negative status if the arguments are invalid). Needs the
 * current device: the tensor-core variant is prepared (not launched) to
 * check that it fits this build. */
int mj_decode_kernel(const mj_decode_args* args);

/* How many mj_decode calls of this process ran the CUDA-core kernel on
 * arguments the tensor-core kernel takes, because no tensor-core variant's
 * register split fits the build (0 on a correct build; the first such call
 * also prints one line on stderr). */
int mj_tc_fallbacks(void);

/* LSE merge of the partials of every sequence with n_splits > 1 into O / LSE. */
int mj_combine(const mj_decode_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* Split-KV planning on the host, and a runner handle that owns a decode's   */
/* plan buffers, for hosts that drive the library without the Python runner. */
/*                                                                            */
/* mj_plan_split_kv replaces arch/thor/plan.py:140-197 `plan_split_kv` (plus */
/* the B200 rebalance, rebalance != 0; item_overhead in tiles, 2.0 is the     */
/* measured per-job cost): sequence lengths in, the work list (seq,          */
/* tile_begin, tile_end, split) of 128-row tiles longest first and each      */
/* sequence's split count out; pad_to > 0 pads the list with empty items.     */
/* Pure host code, no CUDA call.                                             */
int mj_plan_split_kv(const int32_t* seq_lens, int num_seqs, int h_k, int n_q_tiles, int sm_count, int ctas_per_sm,
                     int max_splits, int pad_to, int rebalance, float item_overhead, int32_t* work_out,
                     int work_capacity, int32_t* n_splits_out, int* num_work_out, int* chunk_tiles_out);

/* The runner replaces the reference's T5DecodeRunner state                  */
/* (arch/thor/runner.py:143-174, plan :184-234): mj_create allocates, on     */
/* `device`, the fixed-address work list and split counts (a CUDA graph      */
/* captured on one plan replays any later one), the split partials for       */
/* max_splits x max_num_seqs x h_k x max_q_len x h_q / h_k rows, the status  */
/* word and a pinned staging copy; NULL on failure (see mj_last_error).       */
/* mj_plan plans host sequence lengths (+ margin tokens each) and copies the */
/* plan asynchronously on `stream`; fixed_grid != 0 launches the padded      */
/* capacity (graph capture). mj_runner_fill writes the plan's and buffers'   */
/* fields (shapes, work, n_splits, num_work, partials, part_seqs, status,    */
/* with_combine) into a mj_decode_args whose tensors the caller sets.         */
/* mj_runner_status reads and clears the device status word (synchronous;   */
/* returns MJ_DEV_* or a negative MJ_ERR_*). Calls on one runner are not     */
/* thread-safe.                                                               */
typedef struct mj_runner mj_runner;
mj_runner* mj_create(int device, int h_q, int h_k, int head_size, int page_size, int max_num_seqs, int max_q_len,
                     int kv_format, int max_splits, int ctas_per_sm);
int mj_plan(mj_runner* runner, const int32_t* seq_lens_host, int num_seqs, int q_len, int margin, int fixed_grid,
            void* stream);
int mj_runner_fill(const mj_runner* runner, mj_decode_args* args);
int mj_runner_status(mj_runner* runner);
void mj_destroy(mj_runner* runner);

/* ------------------------------------------------------------------------ */
/* Narrow -> e4m3 page expansion for steps a stock fallback backend runs on */
/* a narrow cache. Replaces kvfp6.py:257-335 `expand_pages_to_fp8` (called   */
/* from backend.py:573-607 on the page map of builder.py:479-509). Output    */
/* page j (0 <= j < num_out_pages) receives the K and V rows of cache page   */
/* src_pages[j]: each e4m3 byte = e4m3(code_value * ratio) with the fp32      */
/* product rounded to nearest even and saturated at +-448 (ratio = 1 when    */
/* the pointer is null, which gives e2m3 / e2m1 values exactly). nvfp4: the */
/* code value is e4m3(code * scale * 2^-3), the value its tensor-core MMA    */
/* reads, then times the ratio as above. A src page outside [0, num_pages)  */
/* flags MJ_DEV_BAD_PAGE and its output page is left untouched. Alignment:  */
/* packed rows 4-byte aligned, output rows 16-byte.                          */
typedef struct mj_expand_args {
  const void* k_cache;          /* narrow logical (num_pages, page_size, h_k, row_bytes) */
  const void* v_cache;
  int64_t k_stride_page, k_stride_row, k_stride_head; /* bytes */
  int64_t v_stride_page, v_stride_row, v_stride_head; /* bytes */
  int64_t num_pages;
  int page_size, h_k, head_size; /* head_size a multiple of 16 */
  const int32_t* src_pages;     /* (num_out_pages,) */
  int64_t num_out_pages;
  void* k_out;                  /* e4m3 logical (>= num_out_pages, page_size, h_k, head_size) */
  void* v_out;
  int64_t ko_stride_page, ko_stride_row, ko_stride_head; /* bytes */
  int64_t vo_stride_page, vo_stride_row, vo_stride_head; /* bytes */
  const float* k_ratio;         /* optional, per k_ratio_mode */
  int k_ratio_mode;             /* MJ_SCALE_TENSOR | _HEAD | _CHANNEL */
  const float* v_ratio;
  int v_ratio_mode;
  int32_t* status;              /* optional device status word (MJ_DEV_*) */
  int kv_format;                /* MJ_KV_E2M3 | _E3M2 | _E2M1 | _NVFP4 */
  const void* k_scales;         /* nvfp4 only: (num_pages, page_size, h_k, head_size / 16) bytes */
  const void* v_scales;
  int64_t ks_stride_page, ks_stride_row, ks_stride_head; /* bytes */
  int64_t vs_stride_page, vs_stride_row, vs_stride_head; /* bytes */
} mj_expand_args;

int mj_expand_pages(const mj_expand_args* args, void* stream);

/* mj_decode for callers that cannot allocate device memory. No counterpart
 * in the reference. Engines that pre-size all of HBM into their own pools,
 * code issuing work during a global-mode stream capture (where cudaMalloc is
 * illegal) and plugin hosts that pass only inputs and outputs cannot supply
 * o_part / lse_part; this entry point ignores those fields (and part_seqs)
 * and keeps the partials in a 16 MiB device array built into the library,
 * which every GPU that loads the library holds until exit. It allocates
 * nothing. The merge always runs inside the call (with_combine is forced on).
 * Limit: max_splits * num_seqs * h_k * (q_len * h_q / h_k) * (head_size + 1)
 * * 4 bytes <= 16 MiB, else MJ_ERR_UNSUPPORTED with a message. The first call
 * on each device looks the array up (cudaGetSymbolAddress) -- make it before
 * any stream capture; the address found stays valid until the device or its
 * primary context is reset (after a reset, do not call this again). All
 * calls on a device share the array and it keeps the last call's contents
 * (nothing in it needs to start at zero); calls that overlap on the GPU
 * race on it and must be ordered. */
int mj_decode_noalloc(const mj_decode_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MJOLNIR_B200_H */
