// C ABI of libmjolnir_b200: argument validation, error reporting, dispatch.
// Every entry point returns an int status and never aborts; the message of
// the last failure of the calling thread is available from mj_last_error().
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

#include "common.cuh"

namespace mj {
cudaError_t launch_cache_write(const mj_cache_write_args& a, cudaStream_t stream);
cudaError_t launch_decode_simt(const mj_decode_args& a, cudaStream_t stream);
cudaError_t launch_combine(const mj_decode_args& a, cudaStream_t stream);
cudaError_t launch_decode_tc(const mj_decode_args& a, cudaStream_t stream, bool* handled, bool dry);
const char* tc_ineligible(const mj_decode_args& a);
cudaError_t launch_expand_pages(const mj_expand_args& a, cudaStream_t stream);
}  // namespace mj

static thread_local char g_err[512] = "";

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) {
    g_err[0] = 0;
    return MJ_OK;
  }
  return fail(MJ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

static bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p % a) == 0; }

namespace mj {
// Lets other translation units of the library report through mj_last_error().
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("MJOLNIR_PDL");
    return !(v && v[0] == '0' && v[1] == 0);
  }();
  return on;
}
}  // namespace mj

extern "C" {

const char* mj_last_error(void) { return g_err; }

int mj_abi_version(void) { return MJ_ABI_VERSION; }

int mj_row_bytes(int head_size, int kv_format) {
  if (head_size <= 0 || head_size % 16) return -1;
  if (kv_format == MJ_KV_FP8_E4M3) return head_size;
  if (kv_format == MJ_KV_E2M3 || kv_format == MJ_KV_E3M2) return head_size * 3 / 4;
  if (kv_format == MJ_KV_E2M1 || kv_format == MJ_KV_NVFP4) return head_size / 2;
  return -1;
}

// nvfp4 scale tensors: present, and (for the tensor-core kernel's 8-byte
// copies) with 8-byte aligned rows when `align8`.
static const char* nvfp4_scales_problem(const void* ks, const void* vs, const int64_t* strides, bool align8) {
  if (!ks || !vs) return "nvfp4 needs k_scales and v_scales";
  if (align8) {
    if (!aligned(ks, 8) || !aligned(vs, 8)) return "nvfp4 scale rows must be 8-byte aligned";
    for (int i = 0; i < 6; ++i)
      if (strides[i] % 8) return "nvfp4 scale strides must be multiples of 8 bytes";
  }
  return nullptr;
}

int mj_cache_write(const mj_cache_write_args* args, void* stream) {
  if (!args) return fail(MJ_ERR_INVALID, "mj_cache_write: null args");
  const mj_cache_write_args& a = *args;
  if (a.num_tokens < 0 || a.h_k <= 0) return fail(MJ_ERR_INVALID, "mj_cache_write: num_tokens %lld h_k %d", (long long)a.num_tokens, a.h_k);
  if (a.num_tokens == 0) {
    g_err[0] = 0;
    return MJ_OK;
  }
  const int rb = mj_row_bytes(a.head_size, a.kv_format);
  if (rb < 0) return fail(MJ_ERR_UNSUPPORTED, "mj_cache_write: head_size %d / kv_format %d", a.head_size, a.kv_format);
  if (a.src_dtype < MJ_DT_BF16 || a.src_dtype > MJ_DT_FP32) return fail(MJ_ERR_INVALID, "mj_cache_write: src_dtype %d", a.src_dtype);
  if (!a.key || !a.value || !a.k_cache || !a.v_cache || !a.slot_mapping || !a.k_scale || !a.v_scale)
    return fail(MJ_ERR_INVALID, "mj_cache_write: null pointer argument");
  if (a.page_size <= 0 || a.num_pages <= 0) return fail(MJ_ERR_INVALID, "mj_cache_write: page_size %d num_pages %lld", a.page_size, (long long)a.num_pages);
  for (int m : {a.k_scale_mode, a.v_scale_mode})
    if (m != MJ_SCALE_TENSOR && m != MJ_SCALE_HEAD && m != MJ_SCALE_CHANNEL)
      return fail(MJ_ERR_INVALID, "mj_cache_write: scale mode %d", m);
  if (a.num_tokens * a.h_k > (int64_t)INT32_MAX / 32) return fail(MJ_ERR_UNSUPPORTED, "mj_cache_write: too many rows");
  if (a.kv_format == MJ_KV_NVFP4) {
    if (a.head_size % 128) return fail(MJ_ERR_UNSUPPORTED, "mj_cache_write: nvfp4 head_size %d (a multiple of 128)", a.head_size);
    if (a.k_scale_mode == MJ_SCALE_CHANNEL || a.v_scale_mode == MJ_SCALE_CHANNEL)
      return fail(MJ_ERR_INVALID, "mj_cache_write: the nvfp4 global scale is per tensor or per KV head");
    const int64_t st[6] = {a.ks_stride_page, a.ks_stride_row, a.ks_stride_head, a.vs_stride_page, a.vs_stride_row, a.vs_stride_head};
    if (const char* why = nvfp4_scales_problem(a.k_scales, a.v_scales, st, false))
      return fail(MJ_ERR_INVALID, "mj_cache_write: %s", why);
  }
  return cuda_status(mj::launch_cache_write(a, (cudaStream_t)stream), "mj_cache_write launch");
}

static int validate_decode(const mj_decode_args& a, const char* who) {
  if (a.num_seqs < 0 || a.q_len < 1 || a.h_k <= 0 || a.h_q <= 0 || a.h_q % a.h_k)
    return fail(MJ_ERR_INVALID, "%s: num_seqs %d q_len %d h_q %d h_k %d", who, a.num_seqs, a.q_len, a.h_q, a.h_k);
  if (a.head_size != 128 && a.head_size != 256)
    return fail(MJ_ERR_UNSUPPORTED, "%s: head_size %d (128 or 256)", who, a.head_size);
  if (a.kv_format < MJ_KV_FP8_E4M3 || a.kv_format > MJ_KV_NVFP4)
    return fail(MJ_ERR_INVALID, "%s: kv_format %d", who, a.kv_format);
  if (a.kv_format == MJ_KV_NVFP4) {
    const int64_t st[6] = {a.ks_stride_page, a.ks_stride_row, a.ks_stride_head, a.vs_stride_page, a.vs_stride_row, a.vs_stride_head};
    if (const char* why = nvfp4_scales_problem(a.k_scales, a.v_scales, st, false))
      return fail(MJ_ERR_INVALID, "%s: %s", who, why);
  }
  const int n_q = a.q_len * (a.h_q / a.h_k);
  if (n_q > 64) return fail(MJ_ERR_UNSUPPORTED, "%s: q_len * h_q / h_k = %d > 64 rows per KV head", who, n_q);
  if (a.q_dtype < MJ_DT_BF16 || a.q_dtype > MJ_DT_FP32 || a.o_dtype < MJ_DT_BF16 || a.o_dtype > MJ_DT_FP32)
    return fail(MJ_ERR_INVALID, "%s: q_dtype %d o_dtype %d", who, a.q_dtype, a.o_dtype);
  if (!a.q || !a.o || !a.k_cache || !a.v_cache || !a.block_table || !a.seq_lens || !a.work || !a.n_splits)
    return fail(MJ_ERR_INVALID, "%s: null pointer argument", who);
  if (a.page_size <= 0 || a.num_pages <= 0 || a.num_work < 0 || a.max_splits < 1)
    return fail(MJ_ERR_INVALID, "%s: page_size %d num_pages %lld num_work %d max_splits %d", who, a.page_size,
                (long long)a.num_pages, a.num_work, a.max_splits);
  const int64_t st[6] = {a.k_stride_page, a.k_stride_row, a.k_stride_head, a.v_stride_page, a.v_stride_row, a.v_stride_head};
  for (int i = 0; i < 6; ++i)
    if (st[i] < 0 || st[i] % 16) return fail(MJ_ERR_UNSUPPORTED, "%s: KV byte strides must be 16-byte multiples", who);
  if (!aligned(a.k_cache, 16) || !aligned(a.v_cache, 16)) return fail(MJ_ERR_UNSUPPORTED, "%s: KV views must be 16-byte aligned", who);
  if (!aligned(a.work, 16)) return fail(MJ_ERR_INVALID, "%s: work list must be 16-byte aligned", who);
  for (int m : {a.k_descale_mode, a.v_descale_mode})
    if (m != MJ_SCALE_TENSOR && m != MJ_SCALE_HEAD && m != MJ_SCALE_SEQ_HEAD)
      return fail(MJ_ERR_INVALID, "%s: descale mode %d", who, m);
  if (a.o_part && (!a.lse_part || a.part_seqs < a.num_seqs))
    return fail(MJ_ERR_INVALID, "%s: partial buffers need lse_part and part_seqs >= num_seqs", who);
  if (a.kernel < MJ_KERNEL_AUTO || a.kernel > MJ_KERNEL_TC) return fail(MJ_ERR_INVALID, "%s: kernel %d", who, a.kernel);
  if (a.kernel == MJ_KERNEL_TC && mj::tc_ineligible(a))
    return fail(MJ_ERR_UNSUPPORTED, "%s: the tensor-core kernel cannot run these arguments (%s)", who, mj::tc_ineligible(a));
  return MJ_OK;
}

int mj_decode_kernel(const mj_decode_args* args) {
  if (!args) return -fail(MJ_ERR_INVALID, "mj_decode_kernel: null args");
  int rc = validate_decode(*args, "mj_decode_kernel");
  if (rc) return -rc;
  if (args->kernel == MJ_KERNEL_SIMT || mj::tc_ineligible(*args)) return MJ_KERNEL_SIMT;
  // prepare the variant mj_decode would launch, without launching it
  bool handled = false;
  const cudaError_t e = mj::launch_decode_tc(*args, nullptr, &handled, true);
  if (e != cudaSuccess) return -cuda_status(e, "mj_decode_kernel (tensor-core variant)");
  return handled ? MJ_KERNEL_TC : MJ_KERNEL_SIMT;
}

int mj_decode(const mj_decode_args* args, void* stream) {
  if (!args) return fail(MJ_ERR_INVALID, "mj_decode: null args");
  const mj_decode_args& a = *args;
  int rc = validate_decode(a, "mj_decode");
  if (rc) return rc;
  if (a.num_seqs == 0 || a.num_work == 0) {
    g_err[0] = 0;
    return MJ_OK;
  }
  cudaStream_t s = (cudaStream_t)stream;
  bool handled = false;
  cudaError_t e = cudaSuccess;
  if (a.kernel != MJ_KERNEL_SIMT) {
    e = mj::launch_decode_tc(a, s, &handled, false);
    if (e != cudaSuccess) return cuda_status(e, "mj_decode launch (tensor-core kernel)");
  }
  if (!handled) {
    e = mj::launch_decode_simt(a, s);
    if (e != cudaSuccess) return cuda_status(e, "mj_decode launch");
  }
  // the one-warpgroup tensor-core variants (every head_dim-256 one) merge in
  // the kernel when given counters
  const bool merged = handled && a.merge_counters && (a.q_len * (a.h_q / a.h_k) <= 16 || a.head_size == 256) &&
                      a.max_splits <= 16;
  if (a.with_combine && !merged) {
    if (!a.o_part) return fail(MJ_ERR_INVALID, "mj_decode: with_combine needs partial buffers");
    return cuda_status(mj::launch_combine(a, s), "mj_combine launch");
  }
  g_err[0] = 0;
  return MJ_OK;
}

int mj_combine(const mj_decode_args* args, void* stream) {
  if (!args) return fail(MJ_ERR_INVALID, "mj_combine: null args");
  const mj_decode_args& a = *args;
  int rc = validate_decode(a, "mj_combine");
  if (rc) return rc;
  if (!a.o_part) return fail(MJ_ERR_INVALID, "mj_combine: null partial buffers");
  if (a.num_seqs == 0) {
    g_err[0] = 0;
    return MJ_OK;
  }
  return cuda_status(mj::launch_combine(a, (cudaStream_t)stream), "mj_combine launch");
}

int mj_expand_pages(const mj_expand_args* args, void* stream) {
  if (!args) return fail(MJ_ERR_INVALID, "mj_expand_pages: null args");
  const mj_expand_args& a = *args;
  if (a.num_out_pages < 0 || a.h_k <= 0 || a.page_size <= 0 || a.num_pages <= 0)
    return fail(MJ_ERR_INVALID, "mj_expand_pages: num_out_pages %lld h_k %d page_size %d num_pages %lld",
                (long long)a.num_out_pages, a.h_k, a.page_size, (long long)a.num_pages);
  if (a.head_size <= 0 || a.head_size % 16)
    return fail(MJ_ERR_UNSUPPORTED, "mj_expand_pages: head_size %d (a multiple of 16)", a.head_size);
  if (a.kv_format < MJ_KV_E2M3 || a.kv_format > MJ_KV_NVFP4)
    return fail(MJ_ERR_INVALID, "mj_expand_pages: kv_format %d (a narrow format)", a.kv_format);
  if (a.kv_format == MJ_KV_NVFP4) {
    const int64_t st[6] = {a.ks_stride_page, a.ks_stride_row, a.ks_stride_head, a.vs_stride_page, a.vs_stride_row, a.vs_stride_head};
    if (const char* why = nvfp4_scales_problem(a.k_scales, a.v_scales, st, false))
      return fail(MJ_ERR_INVALID, "mj_expand_pages: %s", why);
  }
  if (a.num_out_pages == 0) {
    g_err[0] = 0;
    return MJ_OK;
  }
  if (!a.k_cache || !a.v_cache || !a.k_out || !a.v_out || !a.src_pages)
    return fail(MJ_ERR_INVALID, "mj_expand_pages: null pointer argument");
  for (int m : {a.k_ratio_mode, a.v_ratio_mode})
    if (m != MJ_SCALE_TENSOR && m != MJ_SCALE_HEAD && m != MJ_SCALE_CHANNEL)
      return fail(MJ_ERR_INVALID, "mj_expand_pages: ratio mode %d", m);
  const int64_t in_strides[6] = {a.k_stride_page, a.k_stride_row, a.k_stride_head,
                                 a.v_stride_page, a.v_stride_row, a.v_stride_head};
  const int64_t out_strides[6] = {a.ko_stride_page, a.ko_stride_row, a.ko_stride_head,
                                  a.vo_stride_page, a.vo_stride_row, a.vo_stride_head};
  bool ok = aligned(a.k_cache, 4) && aligned(a.v_cache, 4) && aligned(a.k_out, 16) && aligned(a.v_out, 16);
  for (int i = 0; i < 6; ++i) ok = ok && in_strides[i] % 4 == 0 && out_strides[i] % 16 == 0;
  if (!ok) return fail(MJ_ERR_UNSUPPORTED, "mj_expand_pages: packed rows must be 4-byte and output rows 16-byte aligned");
  if (a.num_out_pages * a.page_size * a.h_k > (int64_t)INT32_MAX)
    return fail(MJ_ERR_UNSUPPORTED, "mj_expand_pages: too many rows");
  return cuda_status(mj::launch_expand_pages(a, (cudaStream_t)stream), "mj_expand_pages launch");
}

}  // extern "C"
