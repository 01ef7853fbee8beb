// Paged split-KV decode attention on the CUDA cores (fp32 math).
//
// One CTA of 128 threads per (work item, KV head); a work item is a contiguous
// chunk [tile_begin, tile_end) of 128-row KV tiles of one sequence (the
// planner's unit, plan_split_kv in arch/thor/plan.py:140-197). The CTA serves
// every query row n = qi * h_r + r of the KV head's GQA group and of all
// q_len draft positions from ONE read of each KV row (the reference's row
// packing, quant.py:87-100), with an online softmax in base 2.
//
// Per 128-row tile: thread t dequantizes KV row t (K into registers for the
// dot products, V into a half-precision SMEM tile -- exact for every KV format
// codes), the scores go through SMEM for the row-wise max / exp, and thread t
// accumulates output column(s) t (+128) for every query row.
//
// This is the simple, exact-arithmetic path; the tensor-core kernel
// (decode_tc.cu) is the bandwidth path and is checked against the same oracle.
#pragma once

#include <math.h>

#include <atomic>

#include "common.cuh"

namespace mj {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kSimtMaxDevices = 64;

// 16 consecutive KV codes of a row starting at element c0 -> floats (nvfp4:
// the e4m3 values the tensor cores multiply, from the row's scale bytes).
template <int FMT>
__device__ __forceinline__ void load_codes16(const uint8_t* row, int c0, float* out, const uint8_t* srow = nullptr) {
  if (FMT == MJ_KV_FP8_E4M3) {
    uint4 raw = *reinterpret_cast<const uint4*>(row + c0);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] & 0xFFFFu), __NV_E4M3);
      __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> 16), __NV_E4M3);
      float2 a = __half22float2(__half2(lo));
      float2 b = __half22float2(__half2(hi));
      out[4 * i + 0] = a.x;
      out[4 * i + 1] = a.y;
      out[4 * i + 2] = b.x;
      out[4 * i + 3] = b.y;
    }
  } else if (FMT == MJ_KV_E2M1 || FMT == MJ_KV_NVFP4) {
    // 16 codes = 8 bytes at byte offset c0 / 2 (8-byte aligned), low nibble first
    const uint2 w = *reinterpret_cast<const uint2*>(row + (c0 >> 1));
    if (FMT == MJ_KV_NVFP4) {
      const uint8_t sb = srow[c0 >> 4];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        out[k] = e4m3_value(nvfp4_byte((w.x >> (4 * k)) & 15u, sb));
        out[8 + k] = e4m3_value(nvfp4_byte((w.y >> (4 * k)) & 15u, sb));
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        out[k] = e2m1_value((w.x >> (4 * k)) & 15u);
        out[8 + k] = e2m1_value((w.y >> (4 * k)) & 15u);
      }
    }
  } else {
    // 16 codes = 12 bytes at byte offset c0 * 3 / 4 (4-byte aligned)
    const uint32_t* p = reinterpret_cast<const uint32_t*>(row + (c0 >> 2) * 3);
    const uint32_t w0 = p[0], w1 = p[1], w2 = p[2];
    const uint32_t g[4] = {w0 & 0xFFFFFFu, (w0 >> 24) | ((w1 & 0xFFFFu) << 8),
                           (w1 >> 16) | ((w2 & 0xFFu) << 16), w2 >> 8};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t code = (g[i] >> (6 * k)) & 63u;
        out[4 * i + k] = FMT == MJ_KV_E2M3 ? e2m3_value(code) : e3m2_value(code);
      }
    }
  }
}

template <int D, int NQ>
struct SimtSmem {
  float q[NQ][D];
  float p[NQ][kTileRows];
  __half v[kTileRows][D];
  float corr[NQ];
  float m[NQ];
  float l[NQ];
};

template <int D, int NQ, int FMT>
__global__ void __launch_bounds__(128) decode_simt_kernel(const mj_decode_args a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SimtSmem<D, NQ>& sm = *reinterpret_cast<SimtSmem<D, NQ>*>(smem_raw);
  griddep_wait();  // the cache write before it (PDL launch)
  if (a.with_combine) griddep_launch_dependents();  // the combine may queue up behind this grid
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int4 wi = reinterpret_cast<const int4*>(a.work)[blockIdx.x];
  const int seq = wi.x, tb = wi.y, te = wi.z, split = wi.w;
  if (tb >= te) return;
  const int h = blockIdx.y;
  const int h_k = a.h_k, h_r = a.h_q / a.h_k, q_len = a.q_len;
  const int n_q = q_len * h_r;
  const int L = a.seq_lens[seq];
  const float kd = descale_at(a.k_descale, a.k_descale_mode, seq, h, h_k);
  const float vd = descale_at(a.v_descale, a.v_descale_mode, seq, h, h_k);
  const float c2 = a.softmax_scale * kd * kLog2e;

  // Q rows of this GQA group, pre-multiplied by q_mul and the log2 score scale.
  for (int idx = tid; idx < NQ * D; idx += 128) {
    const int r = idx / D, c = idx % D;
    float v = 0.f;
    if (r < n_q) {
      const int qi = r / h_r, rr = r % h_r;
      const int64_t tok = (int64_t)seq * q_len + qi;
      const int qh = h * h_r + rr;
      v = load_elem(a.q, tok * a.q_stride_tok + qh * a.q_stride_head + c, a.q_dtype);
      if (a.q_mul) v *= a.q_mul[(int64_t)qh * D + c];
      v *= c2;
    }
    sm.q[r][c] = v;
  }

  constexpr int CPT = D / 128;  // output columns per thread
  float acc[NQ][CPT];
  float mreg[NQ / 4], lreg[NQ / 4];
#pragma unroll
  for (int r = 0; r < NQ; ++r)
#pragma unroll
    for (int cc = 0; cc < CPT; ++cc) acc[r][cc] = 0.f;
#pragma unroll
  for (int k = 0; k < NQ / 4; ++k) {
    mreg[k] = -INFINITY;
    lreg[k] = 0.f;
  }
  __syncthreads();

  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.k_cache) + (int64_t)h * a.k_stride_head;
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.v_cache) + (int64_t)h * a.v_stride_head;
  const int32_t* bt = a.block_table + (int64_t)seq * a.block_table_stride;

  for (int tile = tb; tile < te; ++tile) {
    const int j = tile * kTileRows + tid;
    bool valid = j < L;
    int64_t pg = 0;
    if (valid) {
      pg = bt[j / a.page_size];
      if (pg < 0 || pg >= a.num_pages) {
        flag(a.status, MJ_DEV_BAD_PAGE);
        valid = false;
      }
    }
    const int prow = j % a.page_size;
    float s[NQ];
#pragma unroll
    for (int r = 0; r < NQ; ++r) s[r] = 0.f;
    if (valid) {
      const uint8_t* krow = kbase + pg * a.k_stride_page + (int64_t)prow * a.k_stride_row;
      const uint8_t* ksrow = FMT == MJ_KV_NVFP4 ? reinterpret_cast<const uint8_t*>(a.k_scales) + pg * a.ks_stride_page +
                                                     (int64_t)prow * a.ks_stride_row + (int64_t)h * a.ks_stride_head
                                               : nullptr;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 16) {
        float kv[16];
        load_codes16<FMT>(krow, c0, kv, ksrow);
#pragma unroll
        for (int r = 0; r < NQ; ++r) {
          if (r < n_q) {
            float t = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) t = fmaf(sm.q[r][c0 + i], kv[i], t);
            s[r] += t;
          }
        }
      }
      const uint8_t* vrow = vbase + pg * a.v_stride_page + (int64_t)prow * a.v_stride_row;
      const uint8_t* vsrow = FMT == MJ_KV_NVFP4 ? reinterpret_cast<const uint8_t*>(a.v_scales) + pg * a.vs_stride_page +
                                                     (int64_t)prow * a.vs_stride_row + (int64_t)h * a.vs_stride_head
                                               : nullptr;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 16) {
        float vv[16];
        load_codes16<FMT>(vrow, c0, vv, vsrow);
#pragma unroll
        for (int i = 0; i < 16; ++i) sm.v[tid][c0 + i] = __float2half_rn(vv[i]);
      }
    } else {
      for (int c = 0; c < D; ++c) sm.v[tid][c] = __float2half_rn(0.f);
    }
#pragma unroll
    for (int r = 0; r < NQ; ++r) {
      if (r < n_q) {
        const int lim = a.causal ? (L - q_len + r / h_r) : (L - 1);
        sm.p[r][tid] = (valid && j <= lim) ? s[r] : -INFINITY;
      }
    }
    __syncthreads();

    // online softmax: warp w owns query rows w, w + 4, ...
#pragma unroll
    for (int k = 0; k < NQ / 4; ++k) {
      const int r = warp + 4 * k;
      if (r < n_q) {
        float x[4];
        float tmax = -INFINITY;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          x[i] = sm.p[r][lane + 32 * i];
          tmax = fmaxf(tmax, x[i]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
        const float m_old = mreg[k];
        const float m_new = fmaxf(m_old, tmax);
        float corr = 1.f, tsum = 0.f;
        if (m_new != -INFINITY) {
          corr = exp2f(m_old - m_new);  // m_old = -inf -> 0
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float p = exp2f(x[i] - m_new);  // -inf -> 0
            sm.p[r][lane + 32 * i] = p;
            tsum += p;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) sm.p[r][lane + 32 * i] = 0.f;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tsum += __shfl_xor_sync(0xffffffffu, tsum, o);
        lreg[k] = lreg[k] * corr + tsum;
        mreg[k] = m_new;
        if (lane == 0) sm.corr[r] = corr;
      }
    }
    __syncthreads();

#pragma unroll
    for (int r = 0; r < NQ; ++r) {
      if (r < n_q) {
        const float cr = sm.corr[r];
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) acc[r][cc] *= cr;
      }
    }
#pragma unroll 2
    for (int jj = 0; jj < kTileRows; jj += 4) {
      float v[4][CPT];
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int cc = 0; cc < CPT; ++cc) v[u][cc] = __half2float(sm.v[jj + u][tid + 128 * cc]);
#pragma unroll
      for (int r = 0; r < NQ; ++r) {
        if (r < n_q) {
          const float4 p = *reinterpret_cast<const float4*>(&sm.p[r][jj]);
#pragma unroll
          for (int cc = 0; cc < CPT; ++cc) {
            float t = acc[r][cc];
            t = fmaf(p.x, v[0][cc], t);
            t = fmaf(p.y, v[1][cc], t);
            t = fmaf(p.z, v[2][cc], t);
            t = fmaf(p.w, v[3][cc], t);
            acc[r][cc] = t;
          }
        }
      }
    }
    __syncthreads();
  }

  // epilogue
#pragma unroll
  for (int k = 0; k < NQ / 4; ++k) {
    const int r = warp + 4 * k;
    if (r < n_q && lane == 0) {
      sm.m[r] = mreg[k];
      sm.l[r] = lreg[k];
    }
  }
  __syncthreads();
  const bool final_out = a.n_splits[seq] <= 1;
  if (!final_out && (split >= a.max_splits || seq >= a.part_seqs || !a.o_part)) {
    if (tid == 0) flag(a.status, MJ_DEV_BAD_SPLIT);
    return;
  }
#pragma unroll
  for (int r = 0; r < NQ; ++r) {
    if (r < n_q) {
      const float l = sm.l[r];
      const float inv = l > 0.f ? vd / l : 0.f;
      const int qi = r / h_r, rr = r % h_r;
      const int64_t tok = (int64_t)seq * q_len + qi;
      const int qh = h * h_r + rr;
#pragma unroll
      for (int cc = 0; cc < CPT; ++cc) {
        const int c = tid + 128 * cc;
        float o = acc[r][cc] * inv;
        if (final_out) {
          if (a.o_mul) o *= a.o_mul[(int64_t)qh * D + c];
          store_elem(a.o, tok * a.o_stride_tok + qh * a.o_stride_head + c, a.o_dtype, o);
        } else {
          a.o_part[((((int64_t)split * a.part_seqs + seq) * h_k + h) * n_q + r) * D + c] = o;
        }
      }
    }
  }
  if (tid < n_q) {
    const int r = tid;
    const float l = sm.l[r];
    const float lse = l > 0.f ? (sm.m[r] + log2f(l)) * kLn2 : -INFINITY;
    if (final_out) {
      if (a.lse) a.lse[((int64_t)seq * q_len + r / h_r) * a.h_q + h * h_r + r % h_r] = lse;
    } else {
      a.lse_part[(((int64_t)split * a.part_seqs + seq) * h_k + h) * n_q + r] = lse;
    }
  }
}

template <int D, int NQ, int FMT>
static cudaError_t launch_simt_t(const mj_decode_args& a, cudaStream_t stream) {
  const size_t smem = sizeof(SimtSmem<D, NQ>);
  // the shared-memory attribute is per device: set it on each device's first launch
  static std::atomic<bool> attr_done[kSimtMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kSimtMaxDevices) return cudaErrorInvalidDevice;
  if (!attr_done[dev].load(std::memory_order_acquire)) {  // idempotent: a race sets it twice
    e = cudaFuncSetAttribute(decode_simt_kernel<D, NQ, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_done[dev].store(true, std::memory_order_release);
  }
  dim3 grid((unsigned)a.num_work, (unsigned)a.h_k);
  return launch_kernel(decode_simt_kernel<D, NQ, FMT>, grid, dim3(128), smem, stream, a);
}

template <int D, int FMT>
static cudaError_t launch_simt_nq(const mj_decode_args& a, int n_q, cudaStream_t stream) {
  if (n_q <= 8) return launch_simt_t<D, 8, FMT>(a, stream);
  if (n_q <= 16) return launch_simt_t<D, 16, FMT>(a, stream);
  if (n_q <= 32) return launch_simt_t<D, 32, FMT>(a, stream);
  return launch_simt_t<D, 64, FMT>(a, stream);
}

// The entry the host side (decode_simt.cu) calls for one KV format.
template <int FMT>
cudaError_t launch_simt_fmt(const mj_decode_args& a, int n_q, cudaStream_t stream) {
  return a.head_size == 128 ? launch_simt_nq<128, FMT>(a, n_q, stream) : launch_simt_nq<256, FMT>(a, n_q, stream);
}

}  // namespace mj
