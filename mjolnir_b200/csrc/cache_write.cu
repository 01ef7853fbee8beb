// Quantize-on-write of new K/V rows into the paged KV cache (reshape_and_cache).
//
// One warp per (token, KV head); each lane owns groups of 4 consecutive
// elements (one packed 24-bit e2m3 word, or 4 e4m3 bytes) for K and for V.
// The write is a few hundred KB per decode step and launch-latency bound, so
// the kernel favours a single small launch over vector width.
//
// Semantics (bit-exact with the reference quantizers; e3m2 / e2m1 as e2m3 on
// their own tables, 4-bit codes packed two per byte, low nibble first):
//   e2m3: kvfp6.py:107-155 (_write_kv_kernel) / quant.py:34-65 -- x / s in fp32
//         (IEEE division), round to nearest, ties to the smaller magnitude,
//         saturate 7.5, no -0, little-endian 4-codes-in-3-bytes packing.
//   fp8 : (x / s) -> e4m3 round-to-nearest-even, saturating at +-448
//         (arch/thor/harness.py:588-590 plus vLLM's saturating write).
//   nvfp4: quant.py:68-84 with the global scale given (s = gs): per 16
//         elements sc = e4m3(min(amax / 6 / gs, 448)), codes e2m1(x / (sc * gs))
//         (0 where sc * gs is 0), scale bytes into the separate scale tensor.
#include "common.cuh"

namespace mj {

__device__ __forceinline__ float scale_of(const float* s, int mode, int h, int c, int d) {
  if (mode == MJ_SCALE_CHANNEL) return s[(int64_t)h * d + c];
  if (mode == MJ_SCALE_HEAD) return s[h];
  return s[0];
}

template <int FMT>
__global__ void __launch_bounds__(256) cache_write_kernel(mj_cache_write_args a) {
  griddep_wait();  // the new rows come from the previous kernel (PDL launch)
  const int warp = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t pair = warp;
  if (pair >= a.num_tokens * a.h_k) return;
  const int64_t t = pair / a.h_k;
  const int h = (int)(pair % a.h_k);
  const int64_t slot = a.slot_mapping[t];
  if (slot < 0) return;  // padding token
  const int64_t page = slot / a.page_size;
  const int64_t row = slot % a.page_size;
  if (page >= a.num_pages) {
    if (lane == 0) flag(a.status, MJ_DEV_BAD_PAGE);
    return;
  }
  const int d = a.head_size;
  const int groups = d >> 2;
#pragma unroll
  for (int side = 0; side < 2; ++side) {
    const void* src = side ? a.value : a.key;
    const int64_t base = side ? (t * a.value_stride_tok + h * a.value_stride_head)
                              : (t * a.key_stride_tok + h * a.key_stride_head);
    const float* sc = side ? a.v_scale : a.k_scale;
    const int mode = side ? a.v_scale_mode : a.k_scale_mode;
    uint8_t* dst = (uint8_t*)(side ? a.v_cache : a.k_cache) +
                   page * (side ? a.v_stride_page : a.k_stride_page) +
                   row * (side ? a.v_stride_row : a.k_stride_row) +
                   h * (side ? a.v_stride_head : a.k_stride_head);
    for (int g = lane; g < groups; g += 32) {
      float x[4], xin[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = 4 * g + i;
        xin[i] = load_elem(src, base + c, a.src_dtype);
        if (FMT != MJ_KV_NVFP4) x[i] = __fdiv_rn(xin[i], scale_of(sc, mode, h, c, d));
      }
      if (FMT == MJ_KV_NVFP4) {
        // a 16-element scale group is 4 consecutive lanes (head_size % 128 == 0,
        // so every lane of the warp takes part in each pass)
        float am = nan_max(nan_max(fabsf(xin[0]), fabsf(xin[1])), nan_max(fabsf(xin[2]), fabsf(xin[3])));
        am = nan_max(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = nan_max(am, __shfl_xor_sync(0xffffffffu, am, 2));
        const float gs = scale_of(sc, mode, h, 0, d);
        float s = __fdiv_rn(__fdiv_rn(am, 6.0f), gs);
        s = s > 448.f ? 448.f : s;  // NaN stays NaN
        const uint8_t sb = e4m3_byte(s);
        const float den = e4m3_value(sb) * gs;
        uint32_t c[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = e2m1_code(den > 0.f ? __fdiv_rn(xin[i], fmaxf(den, 1e-30f)) : 0.f);
        dst[2 * g + 0] = (uint8_t)(c[0] | (c[1] << 4));
        dst[2 * g + 1] = (uint8_t)(c[2] | (c[3] << 4));
        if ((g & 3) == 0) {
          uint8_t* sdst = (uint8_t*)(side ? a.v_scales : a.k_scales) +
                          page * (side ? a.vs_stride_page : a.ks_stride_page) +
                          row * (side ? a.vs_stride_row : a.ks_stride_row) +
                          h * (side ? a.vs_stride_head : a.ks_stride_head);
          sdst[g >> 2] = sb;
        }
      } else if (FMT == MJ_KV_E2M3 || FMT == MJ_KV_E3M2) {
        uint32_t c[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = FMT == MJ_KV_E2M3 ? e2m3_code(x[i]) : e3m2_code(x[i]);
        const uint32_t w = c[0] | (c[1] << 6) | (c[2] << 12) | (c[3] << 18);
        dst[3 * g + 0] = (uint8_t)(w & 0xFFu);
        dst[3 * g + 1] = (uint8_t)((w >> 8) & 0xFFu);
        dst[3 * g + 2] = (uint8_t)((w >> 16) & 0xFFu);
      } else if (FMT == MJ_KV_E2M1) {
        dst[2 * g + 0] = (uint8_t)(e2m1_code(x[0]) | (e2m1_code(x[1]) << 4));
        dst[2 * g + 1] = (uint8_t)(e2m1_code(x[2]) | (e2m1_code(x[3]) << 4));
      } else {
        // A NaN input keeps its sign bit (0x7F / 0xFF) as the reference's host
        // division does; the device division returns a canonical NaN.
#pragma unroll
        for (int i = 0; i < 4; ++i)
          dst[4 * g + i] = isnan(x[i]) ? (uint8_t)(0x7Fu | (signbit(xin[i]) ? 0x80u : 0u)) : e4m3_byte(x[i]);
      }
    }
  }
}

cudaError_t launch_cache_write(const mj_cache_write_args& a, cudaStream_t stream) {
  const int64_t pairs = a.num_tokens * a.h_k;
  const int64_t threads = pairs * 32;
  const unsigned blocks = (unsigned)((threads + 255) / 256);
  // No early trigger: the decode that follows may start only after every
  // CTA of this write has exited, so no CTA of an earlier kernel still waits
  // for resources (shared memory, TMEM) that a starting decode would hold.
  auto kern = cache_write_kernel<MJ_KV_FP8_E4M3>;
  if (a.kv_format == MJ_KV_NVFP4) kern = cache_write_kernel<MJ_KV_NVFP4>;
  else if (a.kv_format == MJ_KV_E2M3) kern = cache_write_kernel<MJ_KV_E2M3>;
  else if (a.kv_format == MJ_KV_E3M2) kern = cache_write_kernel<MJ_KV_E3M2>;
  else if (a.kv_format == MJ_KV_E2M1) kern = cache_write_kernel<MJ_KV_E2M1>;
  return launch_kernel(kern, dim3(blocks), dim3(256), 0, stream, a);
}

}  // namespace mj
