// Host side of the tensor-core decode: eligibility, TMA tensor maps for the
// KV views (one 5-D K|V box per page for the interleaved (pages, h_k,
// page_size, K row | V row) layout, else a 4-D box per operand), and the
// dispatch to the kernel variants, which are compiled once per KV format
// (inst_<format>.cu).
#include <cuda.h>
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace mj {

template <int FMT>
cudaError_t launch_tc_fmt(const mj_decode_args& a, int n_q, bool fused, const CUtensorMap& mk, const CUtensorMap& mv,
                          cudaStream_t stream, bool dry);

std::mutex& tc_init_mutex() {
  static std::mutex m;
  return m;
}

static std::atomic<int64_t> g_tc_fallbacks{0};

}  // namespace mj

namespace mj {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Why the tensor-core kernel cannot run these arguments (nullptr = it can).
const char* tc_ineligible(const mj_decode_args& a) {
  if (a.kv_format == MJ_KV_NVFP4) {  // the scale rows arrive by 8-byte copies
    if (!a.k_scales || !a.v_scales || (uintptr_t)a.k_scales % 8 || (uintptr_t)a.v_scales % 8) return "nvfp4 scale alignment";
    const int64_t ss[6] = {a.ks_stride_page, a.ks_stride_row, a.ks_stride_head, a.vs_stride_page, a.vs_stride_row, a.vs_stride_head};
    for (int i = 0; i < 6; ++i)
      if (ss[i] % 8) return "nvfp4 scale stride alignment";
  }
  if (a.head_size != 128 && a.head_size != 256) return "head_size not 128 or 256";
  if (a.page_size != 16 && a.page_size != 32 && a.page_size != 64 && a.page_size != 128) return "page size";
  if (a.num_pages >= (int64_t)INT32_MAX) return "num_pages";
  const uintptr_t al = a.kv_format == MJ_KV_FP8_E4M3 ? 16 : 32;
  if ((uintptr_t)a.k_cache % al || (uintptr_t)a.v_cache % al) return "KV view alignment";
  const int64_t st[6] = {a.k_stride_page, a.k_stride_row, a.k_stride_head, a.v_stride_page, a.v_stride_row, a.v_stride_head};
  for (int i = 0; i < 6; ++i)
    if (st[i] % (int64_t)al) return "KV stride alignment";
  if (a.k_stride_row == 0 || a.v_stride_row == 0) return "row stride";
  if (!encode_fn()) return "cuTensorMapEncodeTiled unavailable";
  return nullptr;
}

// TMA element type of a KV format: 6-bit codes land 16 per 16-byte slot (12
// packed bytes, 4 padding), 4-bit codes 16 per 16-byte slot (8 and 8).
static CUtensorMapDataType tma_type(int kv_format) {
  if (kv_format == MJ_KV_E2M3 || kv_format == MJ_KV_E3M2) return CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B;
  if (kv_format == MJ_KV_E2M1 || kv_format == MJ_KV_NVFP4) return CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B;
  return CU_TENSOR_MAP_DATA_TYPE_UINT8;
}

// One operand's rows as (codes, page_size rows, h_k, pages) boxes of one
// page; head_dim 256 adds a dimension of the two 128-code halves of a row
// (codes, half, rows, h_k, pages), one box per half.
static bool make_map(CUtensorMap* m, const void* base, int64_t s_page, int64_t s_row, int64_t s_head,
                     const mj_decode_args& a) {
  const bool narrow = a.kv_format != MJ_KV_FP8_E4M3;
  // a dimension of extent 1 never moves its coordinate; give it any legal stride
  const int64_t fill = narrow ? 32 : 16;
  const cuuint64_t sr = (cuuint64_t)(s_row ? s_row : fill), sh = (cuuint64_t)(s_head ? s_head : fill),
                   sp = (cuuint64_t)(s_page ? s_page : fill);
  CUresult r;
  if (a.head_size == 256) {
    cuuint64_t dims[5] = {128, 2, (cuuint64_t)a.page_size, (cuuint64_t)a.h_k, (cuuint64_t)a.num_pages};
    cuuint64_t strides[4] = {(cuuint64_t)mj_row_bytes(128, a.kv_format), sr, sh, sp};
    cuuint32_t box[5] = {128, 1, (cuuint32_t)a.page_size, 1, 1};
    cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    r = encode_fn()(m, tma_type(a.kv_format), 5, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    cuuint64_t dims[4] = {128, (cuuint64_t)a.page_size, (cuuint64_t)a.h_k, (cuuint64_t)a.num_pages};
    cuuint64_t strides[3] = {sr, sh, sp};
    cuuint32_t box[4] = {128, (cuuint32_t)a.page_size, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    r = encode_fn()(m, tma_type(a.kv_format), 4, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  return r == CUDA_SUCCESS;
}

// Persistent launch: one CTA per resident slot (SMs x CTAs per SM), each walking
// the job list (work item, KV head) with a stride of the grid size. The work
// list is longest-first, so the round-robin is a longest-first assignment.
// K and V rows of a page interleaved in one block per (page, KV head): the
// vLLM / reference layout (pages, h_k, page_size, K row | V row). Then one
// 5-D box -- (codes, 8 rows, K|V, row groups, page * h_k + head) -- loads a
// page's K and V at once: half the TMA operations of separate boxes.
static bool fused_layout(const mj_decode_args& a, int64_t* pagehead_stride) {
  const int64_t rb = mj_row_bytes(a.head_size, a.kv_format);
  if ((uintptr_t)a.v_cache != (uintptr_t)a.k_cache + (uintptr_t)rb) return false;
  if (a.k_stride_page != a.v_stride_page || a.k_stride_row != a.v_stride_row || a.k_stride_head != a.v_stride_head)
    return false;
  if (a.page_size % 8 || a.k_stride_row < 2 * rb) return false;
  if (a.h_k > 1) {
    if (a.k_stride_page != (int64_t)a.h_k * a.k_stride_head) return false;
    *pagehead_stride = a.k_stride_head;
  } else {
    *pagehead_stride = a.k_stride_page ? a.k_stride_page : (int64_t)a.page_size * a.k_stride_row;
  }
  return *pagehead_stride >= (int64_t)a.page_size * a.k_stride_row;
}

// head_dim 256: one map per 128-code half of the rows (half 1 starts half a
// row further on), each box the K and V half-rows of one page.
static bool make_map_fused(CUtensorMap* m, const mj_decode_args& a, int64_t pagehead_stride, int half) {
  const int64_t rb = mj_row_bytes(a.head_size, a.kv_format);
  const int64_t heads = a.h_k > 1 ? a.h_k : 1;
  const unsigned char* base = static_cast<const unsigned char*>(a.k_cache) + half * mj_row_bytes(128, a.kv_format);
  cuuint64_t dims[5] = {128, 8, 2, (cuuint64_t)(a.page_size / 8), (cuuint64_t)(a.num_pages * heads)};
  cuuint64_t strides[4] = {(cuuint64_t)a.k_stride_row, (cuuint64_t)rb, (cuuint64_t)(8 * a.k_stride_row),
                           (cuuint64_t)pagehead_stride};
  cuuint32_t box[5] = {128, 8, 2, (cuuint32_t)(a.page_size / 8), 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = encode_fn()(m, tma_type(a.kv_format), 5,
                           const_cast<unsigned char*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static cudaError_t dispatch_nq(const mj_decode_args& a, int n_q, bool fused, const CUtensorMap& mk,
                               const CUtensorMap& mv, cudaStream_t stream, bool dry) {
  switch (a.kv_format) {
    case MJ_KV_E2M3: return launch_tc_fmt<MJ_KV_E2M3>(a, n_q, fused, mk, mv, stream, dry);
    case MJ_KV_E3M2: return launch_tc_fmt<MJ_KV_E3M2>(a, n_q, fused, mk, mv, stream, dry);
    case MJ_KV_E2M1: return launch_tc_fmt<MJ_KV_E2M1>(a, n_q, fused, mk, mv, stream, dry);
    case MJ_KV_NVFP4: return launch_tc_fmt<MJ_KV_NVFP4>(a, n_q, fused, mk, mv, stream, dry);
    default: return launch_tc_fmt<MJ_KV_FP8_E4M3>(a, n_q, fused, mk, mv, stream, dry);
  }
}

// Launch the tensor-core decode when it can run these arguments; *handled
// tells the caller whether it did (with `dry`, whether it would: the variant
// is prepared but not launched). A tensor-map encoding failure is an error.
// When no variant's register split fits this build, the CUDA-core kernel runs
// instead: that is reported once on stderr and counted (mj_tc_fallbacks).
cudaError_t launch_decode_tc(const mj_decode_args& a, cudaStream_t stream, bool* handled, bool dry) {
  *handled = false;
  if (tc_ineligible(a)) return cudaSuccess;
  CUtensorMap mk, mv;
  int64_t ph_stride = 0;
  const bool fused = fused_layout(a, &ph_stride);
  if (fused) {
    if (!make_map_fused(&mk, a, ph_stride, 0)) return cudaErrorInvalidValue;
    if (a.head_size == 256) {
      if (!make_map_fused(&mv, a, ph_stride, 1)) return cudaErrorInvalidValue;
    } else {
      mv = mk;  // unused
    }
  } else if (!make_map(&mk, a.k_cache, a.k_stride_page, a.k_stride_row, a.k_stride_head, a) ||
             !make_map(&mv, a.v_cache, a.v_stride_page, a.v_stride_row, a.v_stride_head, a)) {
    return cudaErrorInvalidValue;
  }
  *handled = true;
  const int n_q = a.q_len * (a.h_q / a.h_k);
  const cudaError_t e = dispatch_nq(a, n_q, fused, mk, mv, stream, dry);
  if (e == cudaErrorNotSupported) {  // no variant's register split fits: the CUDA-core kernel runs
    *handled = false;
    if (!dry && g_tc_fallbacks.fetch_add(1) == 0)
      fprintf(stderr, "mjolnir_b200: no tensor-core decode variant fits this build for %d rows per KV head "
                      "(kv_format %d); running the CUDA-core decode\n", n_q, a.kv_format);
    return cudaSuccess;
  }
  return e;
}

}  // namespace mj

extern "C" int mj_tc_fallbacks(void) { return (int)mj::g_tc_fallbacks.load(); }
