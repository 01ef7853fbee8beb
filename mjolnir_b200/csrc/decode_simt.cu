// Host side of the CUDA-core decode (its kernel variants are compiled once
// per KV format, inst_<format>.cu) and the LSE combine kernel.
#include <math.h>

#include "common.cuh"

namespace mj {

template <int FMT>
cudaError_t launch_simt_fmt(const mj_decode_args& a, int n_q, cudaStream_t stream);

// ---- LSE merge of split partials (one warp per (seq, KV head, query row)) ----
// The reduction of arch/thor/decode.py:1473-1541, on chunk-normalized partials:
// m = max_j lse_j, w_j = exp(lse_j - m), O = sum_j w_j O_j / sum_j w_j,
// lse = m + log(sum_j w_j). Sequences with n_splits <= 1 were written final.
// Lane j holds split j's LSE and weight (splits beyond 32 loop); the O rows are
// read as float4 columns, all splits' loads issued before the sums.
__global__ void __launch_bounds__(128) combine_kernel(const mj_decode_args a) {
  griddep_wait();  // the partials of the decode before it (PDL launch)
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int h_k = a.h_k, h_r = a.h_q / a.h_k, q_len = a.q_len, n_q = q_len * h_r, D = a.head_size;
  if (wid >= (int64_t)a.num_seqs * h_k * n_q) return;
  const int r = (int)(wid % n_q);
  const int h = (int)((wid / n_q) % h_k);
  const int seq = (int)(wid / ((int64_t)n_q * h_k));
  int ns = a.n_splits[seq];
  if (ns <= 1) return;
  if (ns > a.max_splits || seq >= a.part_seqs) {
    if (lane == 0) flag(a.status, MJ_DEV_BAD_SPLIT);
    ns = min(ns, a.max_splits);
    if (seq >= a.part_seqs) return;
  }
  const int64_t stride_split = (int64_t)a.part_seqs * h_k * n_q;
  const int64_t row = ((int64_t)seq * h_k + h) * n_q + r;
  float m = -INFINITY;
  for (int s = lane; s < ns; s += 32) m = fmaxf(m, a.lse_part[s * stride_split + row]);
  m = warp_allmax(m);
  float den = 0.f;
  if (m != -INFINITY)
    for (int s = lane; s < ns; s += 32) den += expf(a.lse_part[s * stride_split + row] - m);
  den = warp_allsum(den);
  const float inv = den > 0.f ? 1.f / den : 0.f;
  const int qi = r / h_r, rr = r % h_r;
  const int64_t tok = (int64_t)seq * q_len + qi;
  const int qh = h * h_r + rr;
  for (int c = 4 * lane; c < D; c += 128) {
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (m != -INFINITY) {
      for (int s0 = 0; s0 < ns; s0 += 32) {
        // this lane's weight for split s0 + lane, shared with the warp
        const float wl = s0 + lane < ns ? expf(a.lse_part[(s0 + lane) * stride_split + row] - m) : 0.f;
        const int nb = min(32, ns - s0);
#pragma unroll 4
        for (int k = 0; k < nb; ++k) {
          const float w = __shfl_sync(0xffffffffu, wl, k);
          const float4 v = *reinterpret_cast<const float4*>(a.o_part + ((s0 + k) * stride_split + row) * D + c);
          o.x = fmaf(w, v.x, o.x);
          o.y = fmaf(w, v.y, o.y);
          o.z = fmaf(w, v.z, o.z);
          o.w = fmaf(w, v.w, o.w);
        }
      }
    }
    const float ov[4] = {o.x * inv, o.y * inv, o.z * inv, o.w * inv};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float v = ov[k];
      if (a.o_mul) v *= a.o_mul[(int64_t)qh * D + c + k];
      store_elem(a.o, tok * a.o_stride_tok + qh * a.o_stride_head + c + k, a.o_dtype, v);
    }
  }
  if (lane == 0 && a.lse) a.lse[tok * a.h_q + qh] = (m != -INFINITY && den > 0.f) ? m + logf(den) : -INFINITY;
}

cudaError_t launch_decode_simt(const mj_decode_args& a, cudaStream_t stream) {
  const int n_q = a.q_len * (a.h_q / a.h_k);
  switch (a.kv_format) {
    case MJ_KV_E2M3: return launch_simt_fmt<MJ_KV_E2M3>(a, n_q, stream);
    case MJ_KV_E3M2: return launch_simt_fmt<MJ_KV_E3M2>(a, n_q, stream);
    case MJ_KV_E2M1: return launch_simt_fmt<MJ_KV_E2M1>(a, n_q, stream);
    case MJ_KV_NVFP4: return launch_simt_fmt<MJ_KV_NVFP4>(a, n_q, stream);
    default: return launch_simt_fmt<MJ_KV_FP8_E4M3>(a, n_q, stream);
  }
}

cudaError_t launch_combine(const mj_decode_args& a, cudaStream_t stream) {
  const int n_q = a.q_len * (a.h_q / a.h_k);
  const int64_t warps = (int64_t)a.num_seqs * a.h_k * n_q;
  if (warps == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((warps * 32 + 127) / 128);
  return launch_kernel(combine_kernel, dim3(blocks), dim3(128), 0, stream, a);
}

}  // namespace mj
