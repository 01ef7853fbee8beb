// Narrow -> e4m3 page expansion: the pages a stock fallback backend reads on a
// narrow (e2m3, e3m2, e2m1, nvfp4) cache, written as e4m3 bytes into its
// scratch cache.
//
// One thread per 16 codes of one row side (12 or 8 packed bytes in, 16 out),
// a grid-stride loop over (out page, row, head, side, chunk) with the chunk
// fastest, so a warp reads 4 consecutive packed rows' worth of contiguous
// bytes and writes 16-byte stores. Pure byte streaming: HBM-bound, a few MB
// per fallback step.
//
// Semantics (kvfp6.py:157-205 `_expand_kernel`, RATIO branch): the e2m3 code
// value times the ratio in fp32, converted to e4m3 with round-to-nearest-even
// and saturation at +-448; without a ratio the byte is the code's exact
// e4m3 encoding (every e2m3 and e2m1 value is representable in e4m3). nvfp4
// codes first become e4m3(code * scale * 2^-3), the tensor cores' value.
#include "common.cuh"

namespace mj {

__device__ __forceinline__ float ratio_at(const float* r, int mode, int h, int c, int d) {
  if (!r) return 1.0f;
  if (mode == MJ_SCALE_CHANNEL) return r[(int64_t)h * d + c];
  if (mode == MJ_SCALE_HEAD) return r[h];
  return r[0];
}

template <int FMT>
__global__ void __launch_bounds__(256) expand_pages_kernel(mj_expand_args a) {
  const int d = a.head_size;
  const int chunks = d >> 4;  // 16 codes per chunk
  const int64_t per_page = (int64_t)a.page_size * a.h_k * 2 * chunks;
  const int64_t total = a.num_out_pages * per_page;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i;
    const int ch = (int)(r % chunks);
    r /= chunks;
    const int side = (int)(r % 2);
    r /= 2;
    const int h = (int)(r % a.h_k);
    r /= a.h_k;
    const int row = (int)(r % a.page_size);
    const int64_t j = r / a.page_size;
    const int32_t src = a.src_pages[j];
    if (src < 0 || (int64_t)src >= a.num_pages) {
      if (row == 0 && h == 0 && side == 0 && ch == 0) flag(a.status, MJ_DEV_BAD_PAGE);
      continue;
    }
    constexpr int IN = (FMT == MJ_KV_E2M1 || FMT == MJ_KV_NVFP4) ? 8 : 12;  // packed bytes of 16 codes
    const uint8_t* in = (const uint8_t*)(side ? a.v_cache : a.k_cache) +
                        (int64_t)src * (side ? a.v_stride_page : a.k_stride_page) +
                        (int64_t)row * (side ? a.v_stride_row : a.k_stride_row) +
                        (int64_t)h * (side ? a.v_stride_head : a.k_stride_head) + ch * IN;
    uint8_t* out = (uint8_t*)(side ? a.v_out : a.k_out) + j * (side ? a.vo_stride_page : a.ko_stride_page) +
                   (int64_t)row * (side ? a.vo_stride_row : a.ko_stride_row) +
                   (int64_t)h * (side ? a.vo_stride_head : a.ko_stride_head) + ch * 16;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(in);
    uint32_t code16[16];
    if constexpr (IN == 12) {
      const uint32_t w0 = w[0], w1 = w[1], w2 = w[2];
      // 4 little-endian 24-bit words of 4 codes each
      const uint32_t word[4] = {w0 & 0xFFFFFFu, (w0 >> 24) | ((w1 & 0xFFFFu) << 8),
                                (w1 >> 16) | ((w2 & 0xFFu) << 16), w2 >> 8};
#pragma unroll
      for (int i = 0; i < 16; ++i) code16[i] = (word[i >> 2] >> (6 * (i & 3))) & 63u;
    } else {
      const uint32_t w0 = w[0], w1 = w[1];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        code16[i] = (w0 >> (4 * i)) & 15u;
        code16[8 + i] = (w1 >> (4 * i)) & 15u;
      }
    }
    uint8_t sb = 0;
    if constexpr (FMT == MJ_KV_NVFP4) {  // the group's scale byte (16 codes = one group)
      sb = *((const uint8_t*)(side ? a.v_scales : a.k_scales) + (int64_t)src * (side ? a.vs_stride_page : a.ks_stride_page) +
             (int64_t)row * (side ? a.vs_stride_row : a.ks_stride_row) +
             (int64_t)h * (side ? a.vs_stride_head : a.ks_stride_head) + ch);
    }
    const float* ratio = side ? a.v_ratio : a.k_ratio;
    const int mode = side ? a.v_ratio_mode : a.k_ratio_mode;
    uint32_t o[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      uint32_t packed = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t code = code16[4 * g + k];
        const int c = ch * 16 + g * 4 + k;
        float v;
        if constexpr (FMT == MJ_KV_E2M3) v = e2m3_value(code);
        else if constexpr (FMT == MJ_KV_E3M2) v = e3m2_value(code);
        else if constexpr (FMT == MJ_KV_E2M1) v = e2m1_value(code);
        else v = e4m3_value(nvfp4_byte(code, sb));
        v *= ratio_at(ratio, mode, h, c, d);
        packed |= (uint32_t)e4m3_byte(v) << (8 * k);
      }
      o[g] = packed;
    }
    *reinterpret_cast<uint4*>(out) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

cudaError_t launch_expand_pages(const mj_expand_args& a, cudaStream_t stream) {
  const int64_t total = a.num_out_pages * a.page_size * a.h_k * 2 * (a.head_size >> 4);
  if (total == 0) return cudaSuccess;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (total + 255) / 256;
  const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  auto kern = expand_pages_kernel<MJ_KV_E2M3>;
  if (a.kv_format == MJ_KV_E3M2) kern = expand_pages_kernel<MJ_KV_E3M2>;
  else if (a.kv_format == MJ_KV_E2M1) kern = expand_pages_kernel<MJ_KV_E2M1>;
  else if (a.kv_format == MJ_KV_NVFP4) kern = expand_pages_kernel<MJ_KV_NVFP4>;
  kern<<<grid, 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace mj
