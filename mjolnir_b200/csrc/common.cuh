// Device helpers shared by the mjolnir_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mjolnir_b200.h"

namespace mj {

constexpr int kTileRows = 128;  // KV rows per work tile (the planner's unit)

// ---- element loads / stores by runtime dtype ------------------------------
__device__ __forceinline__ float load_elem(const void* p, int64_t i, int dt) {
  if (dt == MJ_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dt == MJ_DT_FP16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_elem(void* p, int64_t i, int dt, float v) {
  if (dt == MJ_DT_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dt == MJ_DT_FP16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// warp-wide max / sum, the result in every lane
__device__ __forceinline__ float warp_allmax(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// max that propagates NaN (as torch's amax does)
__device__ __forceinline__ float nan_max(float a, float b) { return (a > b || a != a) ? a : b; }

__device__ __forceinline__ void flag(int32_t* status, int code) {
  if (status) atomicExch(status, code);
}

// ---- e2m3 (sign | 2-bit exp | 3-bit mantissa, bias 1, max 7.5) -----------
// Value of a magnitude code 0..31, from the bit definition: e == 0 -> m / 8,
// else (8 + m) * 2^(e - 1) / 8. Exact in fp32 (and in fp16).
__device__ __forceinline__ float e2m3_mag_value(uint32_t mag) {
  uint32_t e = mag >> 3, m = mag & 7u;
  uint32_t eighths = e ? ((8u + m) << (e - 1u)) : m;
  return (float)eighths * 0.125f;
}

__device__ __forceinline__ float e2m3_value(uint32_t code) {
  float v = e2m3_mag_value(code & 31u);
  return (code & 32u) ? -v : v;
}

// fp32 (already divided by the scale) -> e2m3 code 0..63: round to nearest,
// ties to the smaller magnitude, saturating at 7.5 (NaN -> 7.5), the sign bit
// only for a non-zero magnitude. The neighbour comparison is the reference's
// fp32 expression (ax - lo) <= (hi - ax) (quant.py:43), evaluated with
// explicitly rounded subtractions.
__device__ __forceinline__ uint32_t e2m3_code(float x) {
  float ax = fabsf(x);
  uint32_t mag;
  if (!(ax < 7.5f)) {  // >= 7.5, +-inf or NaN
    mag = 31u;
  } else {
    uint32_t lo;
    float lo_v, step;
    if (ax < 2.0f) {           // codes 0..16, spacing 1/8
      lo = (uint32_t)(ax * 8.0f);
      lo_v = (float)lo * 0.125f;
      step = 0.125f;
    } else if (ax < 4.0f) {    // codes 16..24, spacing 1/4
      uint32_t k = (uint32_t)((ax - 2.0f) * 4.0f);
      lo = 16u + k;
      lo_v = 2.0f + (float)k * 0.25f;
      step = 0.25f;
    } else {                   // codes 24..31, spacing 1/2
      uint32_t k = (uint32_t)((ax - 4.0f) * 2.0f);
      lo = 24u + k;
      lo_v = 4.0f + (float)k * 0.5f;
      step = 0.5f;
    }
    if (ax == lo_v) {
      mag = lo;
    } else {
      float hi_v = lo_v + step;
      bool pick_lo = __fsub_rn(ax, lo_v) <= __fsub_rn(hi_v, ax);
      mag = pick_lo ? lo : lo + 1u;
    }
  }
  uint32_t neg = (x < 0.0f && mag != 0u) ? 32u : 0u;
  return mag | neg;
}

// ---- e3m2 (bias 3, max 28) and e2m1 (bias 1, max 6) ------------------------
// Values from the bit definitions; codes by the same rule as e2m3 (nearest,
// ties to the smaller magnitude, saturating, NaN -> max, no -0). Above the
// subnormal range the lower neighbour is the input truncated to the format's
// mantissa bits and the step one unit of its last place.
__device__ __forceinline__ float e3m2_value(uint32_t code) {
  const uint32_t mag = code & 31u, e = mag >> 2, m = mag & 3u;
  const uint32_t sixteenths = e ? ((4u + m) << (e - 1u)) : m;
  const float v = (float)sixteenths * 0.0625f;
  return (code & 32u) ? -v : v;
}

__device__ __forceinline__ float e2m1_value(uint32_t code) {
  const uint32_t mag = code & 7u, e = mag >> 1, m = mag & 1u;
  const uint32_t halves = e ? ((2u + m) << (e - 1u)) : m;
  const float v = (float)halves * 0.5f;
  return (code & 8u) ? -v : v;
}

// MB mantissa bits, BIAS, EB exponent bits; sub_step = the subnormal spacing.
template <int EB, int MB, int BIAS>
__device__ __forceinline__ uint32_t minifloat_code(float x) {
  constexpr uint32_t kMagMax = (1u << (EB + MB)) - 1u;
  constexpr float kMin = 1.0f / (float)(1u << (BIAS - 1));  // smallest normal: 2^(1 - BIAS)
  const float vmax = (float)((2u << MB) - 1u) / (float)(1u << MB) * (float)(1u << ((1u << EB) - 1u - BIAS));
  const float ax = fabsf(x);
  uint32_t mag;
  if (!(ax < vmax)) {  // >= max, +-inf or NaN
    mag = kMagMax;
  } else {
    uint32_t lo;
    float lo_v, step;
    if (ax < kMin) {  // subnormals: spacing 2^(1 - BIAS - MB)
      const float sub = kMin / (float)(1u << MB);
      lo = (uint32_t)(ax / sub);
      lo_v = (float)lo * sub;
      step = sub;
    } else {
      const uint32_t u = __float_as_uint(ax);
      const int E = (int)(u >> 23) - 127;
      lo = ((uint32_t)(E + BIAS) << MB) | ((u >> (23 - MB)) & ((1u << MB) - 1u));
      lo_v = __uint_as_float(u & ~((1u << (23 - MB)) - 1u));
      step = __uint_as_float((uint32_t)(E - MB + 127) << 23);
    }
    if (ax == lo_v) {
      mag = lo;
    } else {
      const float hi_v = lo_v + step;
      mag = __fsub_rn(ax, lo_v) <= __fsub_rn(hi_v, ax) ? lo : lo + 1u;
    }
  }
  const uint32_t neg = (x < 0.0f && mag) ? (1u << (EB + MB)) : 0u;  // NaN and -0 stay positive
  return mag | neg;
}

__device__ __forceinline__ uint32_t e3m2_code(float x) { return minifloat_code<3, 2, 3>(x); }
__device__ __forceinline__ uint32_t e2m1_code(float x) { return minifloat_code<2, 1, 1>(x); }

// fp32 -> e4m3fn byte: round to nearest even, saturate at +-448, NaN keeps
// its sign bit (0x7F / 0xFF).
__device__ __forceinline__ uint8_t e4m3_byte(float x) {
  if (isnan(x)) return (uint8_t)(0x7Fu | (signbit(x) ? 0x80u : 0u));
  x = fminf(fmaxf(x, -448.0f), 448.0f);
  return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

__device__ __forceinline__ float e4m3_value(uint8_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(__half(h));
}

// nvfp4: the e4m3 byte the tensor cores multiply for e2m1 code `code` of a
// group with scale byte `sb`: e4m3(value(code) * value(sb) * 2^-3). The fp32
// product is exact, so the one rounding is the e4m3 conversion
// (quant.py:81-83).
__device__ __forceinline__ uint8_t nvfp4_byte(uint32_t code, uint8_t sb) {
  return e4m3_byte(e2m1_value(code) * e4m3_value(sb) * 0.125f);
}

// Descale of (seq, head) under a mode.
__device__ __forceinline__ float descale_at(const float* p, int mode, int seq, int h, int h_k) {
  if (!p) return 1.0f;
  if (mode == MJ_SCALE_TENSOR) return p[0];
  if (mode == MJ_SCALE_HEAD) return p[h];
  return p[(int64_t)seq * h_k + h];
}

// ---- programmatic dependent launch (PDL) -----------------------------------
// A kernel launched with programmatic stream serialization may start while
// the previous kernel in the stream is still draining; every thread that reads
// memory the previous kernel wrote first waits here for that grid to complete
// and flush (a no-op for a kernel launched without the attribute).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next PDL-launched kernel be scheduled once every CTA of this grid
// has issued it (or exited); its own griddep_wait still waits for this grid.
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launch with programmatic stream serialization unless MJOLNIR_PDL=0.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace mj
