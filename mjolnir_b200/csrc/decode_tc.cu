// Paged split-KV decode attention on the 5th-generation tensor cores (sm_100a).
//
// One CTA per (work item, KV head); a work item is a contiguous chunk of
// 128-row KV tiles of one sequence (the planner's unit, the reference's
// arch/thor/plan.py:140-197), and the CTA serves all n_q = q_len * h_r query
// rows of the KV head from one read of each KV byte.
//
// Data path per 128-row tile:
//   TMA (one box per page, shuffled pages via the block table) -> SMEM ring,
//   128-byte swizzled; e2m3 rows arrive through the 16U6 TMA type (12 packed
//   bytes per 16-byte slot), e4m3 rows as bytes. Pages past the sequence are
//   read at an out-of-range page coordinate: the TMA zero-fills them.
//   S = K . Q^T        tcgen05.mma kind::f8f6f4, M = 128 KV rows, N = 3*NQP,
//                      A = K (e4m3 or e2m3, K-major), B = Q split in three
//                      e4m3 terms (rows [0,NQP) = hi, [NQP,2NQP) = mid =
//                      (q - hi) * 16, [2NQP,3NQP) = lo = (q - hi - mid/16) * 256)
//   softmax            4 warps, thread = TMEM lane = KV row; base-2 online
//                      softmax in fp32; P split the same way into three e4m3
//                      terms (scaled by 448) and stored K-major for the next MMA
//   O^T = V^T . P^T    tcgen05.mma kind::f8f6f4, M = 128 head-dim rows,
//                      A = V (e4m3, MN-major), B = P; a fresh TMEM tile per KV
//                      tile, folded into fp32 registers (thread = head-dim
//                      lane) with the running-max correction
//   e2m3 V cannot be an MN-major MMA operand, so two converter warps turn each
//   16-code chunk into 16 e4m3 bytes of value code * 2^-6 (exact; the 2^6 is
//   folded into the output scale) at the same swizzled offset.
//
// Numerics: split-fp8 Q and P carry ~12 significant bits each
// (hi + mid / 16 + lo / 256),
// accumulation is fp32 in TMEM, softmax is fp32; the reference's
// single-e4m3 recipe (arch/thor/decode.py:1288-1297) is not used because it
// misses the 2e-3 tolerance.
//
// Every mbarrier wait is bounded (MJ_TC_WAIT_NS); on a timeout the CTA sets
// MJ_DEV_TIMEOUT in the status word, all roles stop at their next wait, wait
// (bounded) for their in-flight copies and MMAs, free TMEM and return.
#include <math.h>

#include "common.cuh"
#include "sm100.cuh"

#ifndef MJ_TC_WAIT_NS
#define MJ_TC_WAIT_NS 500000000ull  // 0.5 s per wait: a tile takes microseconds
#endif

namespace mj {
namespace tc {

using namespace sm100;

constexpr int kThreads = 256;   // 8 warps
constexpr int kTileBytes = 128 * 128;  // one 128 x 128 byte operand tile (e2m3: 16U6 slots)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kPScale = 448.0f;  // P (<= 1) is stored as e4m3(p * 448) hi/lo

// warp roles
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpCvt0 = 2;   // warps 2-3: V conversion (e2m3) / tail zeroing (e4m3)
constexpr int kWarpSm0 = 4;    // warps 4-7: softmax warpgroup

template <int FMT, int NQP>
struct Cfg {
  static constexpr int N = 3 * NQP;                       // MMA N: hi, mid, lo row blocks
  static constexpr int STAGES = (FMT == MJ_KV_E2M3) ? 2 : 3;
  static constexpr int TMEM_COLS = (4 * N) <= 32 ? 32 : (4 * N) <= 64 ? 64 : (4 * N) <= 128 ? 128 : 256;
  static_assert(4 * N <= 256, "two CTAs per SM share the 512 TMEM columns");
  static constexpr uint32_t TX_BYTES = (FMT == MJ_KV_E2M3) ? 2u * 128u * 96u : 2u * 128u * 128u;
  // shared memory plan (offsets from a 1024-aligned base)
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + STAGES * kTileBytes;
  static constexpr int VC_OFF = V_OFF + STAGES * kTileBytes;               // e2m3 converted V ring (2)
  static constexpr int Q_OFF = VC_OFF + ((FMT == MJ_KV_E2M3) ? 2 * kTileBytes : 0);
  static constexpr int P_OFF = Q_OFF + N * 128;                            // P ring (2)
  static constexpr int BAR_OFF = P_OFF + 2 * N * 128;
  static constexpr int NBARS = 2 * STAGES + 2 * 7 + 2;  // full/empty, 7 pairs, q_full, drain
  static constexpr int RED_OFF = BAR_OFF + NBARS * 8;    // float red[2][4][NQP]
  static constexpr int LIM_OFF = RED_OFF + 2 * 4 * NQP * 4;  // int lim[NQP]
  static constexpr int MISC_OFF = LIM_OFF + NQP * 4;     // tmem base, abort flag, l/m scratch
  static constexpr int SMEM = MISC_OFF + 64 + 4 * 4 * NQP + 1024;  // + alignment slack
};

struct Bars {
  uint64_t* full;
  uint64_t* empty;
  uint64_t *s_full, *s_free, *p_full, *o_full, *o_free, *v_ready, *v_free;
  uint64_t* q_full;
  uint64_t* drain;
};

// Turn 16 e2m3 codes (12 packed bytes of a 16U6 slot) into 16 e4m3 bytes whose
// values are the codes' values * 2^-6: sign moves from bit 5 to bit 7, the
// 2-bit exponent and 3-bit mantissa stay (e4m3 bias 7 vs e2m3 bias 1).
__device__ __forceinline__ uint32_t spread4(uint32_t g) {
  uint32_t t = g + 15u * (g & 0xFFF000u);      // c2 c3 -> bits 16..27
  t = t + 3u * (t & 0x0FC00FC0u);              // c1 -> byte 1, c3 -> byte 3
  return t + 3u * (t & 0x20202020u);           // sign bit 5 -> bit 7 in every byte
}

__device__ __forceinline__ uint4 e2m3x16_to_e4m3(uint4 raw) {
  const uint32_t g0 = raw.x & 0xFFFFFFu;
  const uint32_t g1 = __funnelshift_r(raw.x, raw.y, 24) & 0xFFFFFFu;
  const uint32_t g2 = __funnelshift_r(raw.y, raw.z, 16) & 0xFFFFFFu;
  const uint32_t g3 = raw.z >> 8;
  return make_uint4(spread4(g0), spread4(g1), spread4(g2), spread4(g3));
}

// y0, y1 (|y| <= 448) -> three e4m3 terms each: y ~= hi + mid / 16 + lo / 256.
// The residuals are exact in fp32 (hi is within a factor of 2 of y).
__device__ __forceinline__ void split3(float y0, float y1, uint16_t& hb, uint16_t& mb, uint16_t& lb) {
  hb = f2_to_e4m3x2(y0, y1);
  const float2 hv = e4m3x2_to_f2(hb);
  const float r0 = (y0 - hv.x) * 16.f, r1 = (y1 - hv.y) * 16.f;
  mb = f2_to_e4m3x2(r0, r1);
  const float2 mv = e4m3x2_to_f2(mb);
  lb = f2_to_e4m3x2((r0 - mv.x) * 16.f, (r1 - mv.y) * 16.f);
}

// Stores the three-term split of rows r, r+1 (column t) into a K-major tile.
template <int NQP>
__device__ __forceinline__ void store_split(unsigned char* buf, int r, int t, uint16_t hb, uint16_t mb, uint16_t lb) {
  buf[sw128_offset(r, t)] = (uint8_t)(hb & 0xFF);
  buf[sw128_offset(r + 1, t)] = (uint8_t)(hb >> 8);
  buf[sw128_offset(NQP + r, t)] = (uint8_t)(mb & 0xFF);
  buf[sw128_offset(NQP + r + 1, t)] = (uint8_t)(mb >> 8);
  buf[sw128_offset(2 * NQP + r, t)] = (uint8_t)(lb & 0xFF);
  buf[sw128_offset(2 * NQP + r + 1, t)] = (uint8_t)(lb >> 8);
}

// 3*NQP TMEM columns of this thread's lane -> v
template <int NQP>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float* v) {
  constexpr int C = 3 * NQP;
#pragma unroll
  for (int c = 0; c + 16 <= C; c += 16) tmem_ld16(taddr + c, v + c);
  if (C % 16) tmem_ld8(taddr + (C / 16) * 16, v + (C / 16) * 16);
}

template <int NQP>
__device__ __forceinline__ float combine3(const float* v, int r) {
  return v[r] + v[NQP + r] * 0.0625f + v[2 * NQP + r] * 0.00390625f;
}

}  // namespace tc
}  // namespace mj

namespace mj {
namespace tc {

template <int FMT, int NQP>
__global__ void __launch_bounds__(kThreads, 2)
    decode_tc_kernel(const __grid_constant__ mj_decode_args a, const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv) {
  using C = Cfg<FMT, NQP>;
  constexpr int N = C::N;
  constexpr int S = C::STAGES;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int4 wi = reinterpret_cast<const int4*>(a.work)[blockIdx.x];
  const int seq = wi.x, tb = wi.y, te = wi.z, split = wi.w;
  if (tb >= te) return;  // empty (padding) item: uniform exit before any barrier
  const int h = blockIdx.y;
  const int L = a.seq_lens[seq];
  const int n_tiles = te - tb;

  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  Bars b;
  b.full = bars;
  b.empty = bars + S;
  b.s_full = bars + 2 * S;
  b.s_free = b.s_full + 2;
  b.p_full = b.s_free + 2;
  b.o_full = b.p_full + 2;
  b.o_free = b.o_full + 2;
  b.v_ready = b.o_free + 2;
  b.v_free = b.v_ready + 2;
  b.q_full = b.v_free + 2;
  b.drain = b.q_full + 1;
  float* red = reinterpret_cast<float*>(sm + C::RED_OFF);   // [2][4][NQP]
  int* lim_s = reinterpret_cast<int*>(sm + C::LIM_OFF);      // [NQP]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + C::MISC_OFF + 4);
  float* lred = reinterpret_cast<float*>(sm + C::MISC_OFF + 64);  // [4][NQP]
  __shared__ int never_abort;  // a flag no one sets: drains wait on time only

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&b.full[i], 1);
      mbar_init(&b.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b.s_full[i], 1);
      mbar_init(&b.s_free[i], 128);
      mbar_init(&b.p_full[i], 128);
      mbar_init(&b.o_full[i], 1);
      mbar_init(&b.o_free[i], 128);
      mbar_init(&b.v_ready[i], 64);
      mbar_init(&b.v_free[i], 1);
    }
    mbar_init(b.q_full, 1);
    mbar_init(b.drain, 1);
    *abort_flag = 0;
    never_abort = 0;
    fence_mbar_init();
  }
  if (warp == kWarpTma && lane == 0) {
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S0 [0,N) S1 [N,2N) O0 [2N,3N) O1 [3N,4N)

  auto kbuf = [&](int st) { return sm + C::K_OFF + st * kTileBytes; };
  auto vbuf = [&](int st) { return sm + C::V_OFF + st * kTileBytes; };
  auto vcvt = [&](int i) { return sm + C::VC_OFF + i * kTileBytes; };
  unsigned char* qbuf = sm + C::Q_OFF;
  auto pbuf = [&](int i) { return sm + C::P_OFF + i * N * 128; };
  auto give_up = [&]() {
    *abort_flag = 1;
    flag(a.status, MJ_DEV_TIMEOUT);
  };

  if (warp == kWarpTma) {
    // ---------------------------------------------------------------- producer
    const int PS = a.page_size;
    const int P = kTileRows / PS;  // pages per tile; lane p < P loads page p
    const int32_t* bt = a.block_table + (int64_t)seq * a.block_table_stride;
    auto page_coord = [&](int i) {
      int pg = (int)a.num_pages;  // out of range -> the TMA zero-fills the box
      const int row0 = (tb + i) * kTileRows + lane * PS;
      if (lane < P && row0 < L) {
        const int v = bt[row0 / PS];
        if (v < 0 || (int64_t)v >= a.num_pages) {
          flag(a.status, MJ_DEV_BAD_PAGE);
        } else {
          pg = v;
        }
      }
      return pg;
    };
    int pg_next = page_coord(0);
    int issued = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int st = i % S;
      const int pg = pg_next;
      if (i + 1 < n_tiles) pg_next = page_coord(i + 1);
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&b.empty[st], ((i / S) & 1) ^ 1, abort_flag, MJ_TC_WAIT_NS);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        if (lane == 0 && !*abort_flag) give_up();
        break;
      }
      if (lane == 0) mbar_arrive_expect_tx(&b.full[st], C::TX_BYTES);
      __syncwarp();
      if (lane < P) {
        tma_load_4d(kbuf(st) + lane * PS * 128, &tmk, &b.full[st], 0, 0, h, pg);
        tma_load_4d(vbuf(st) + lane * PS * 128, &tmv, &b.full[st], 0, 0, h, pg);
      }
      issued = i + 1;
    }
    // every issued copy must land before the CTA may exit
    if (lane == 0 && *abort_flag) {
      for (int k = issued > S ? issued - S : 0; k < issued; ++k)
        mbar_wait(&b.full[k % S], (k / S) & 1, &never_abort, MJ_TC_WAIT_NS);
    }
    __syncwarp();
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(b.q_full, 0, abort_flag, MJ_TC_WAIT_NS);
      const uint32_t idesc_s = idesc_f8f6f4(FMT == MJ_KV_E2M3 ? 3u : 0u, 0u, 0u, 0u, (uint32_t)N);
      const uint32_t idesc_o = idesc_f8f6f4(0u, 0u, 1u, 0u, (uint32_t)N);
      const uint32_t qaddr = smem_addr(qbuf);
      for (int i = 0; ok && i <= n_tiles; ++i) {
        if (i < n_tiles) {  // S_i = K_i . Q^T
          const int st = i % S;
          ok = mbar_wait(&b.full[st], (i / S) & 1, abort_flag, MJ_TC_WAIT_NS) &&
               mbar_wait(&b.s_free[i & 1], ((i >> 1) & 1) ^ 1, abort_flag, MJ_TC_WAIT_NS);
          if (!ok) break;
          tc_fence_after();
          const uint32_t kaddr = smem_addr(kbuf(st));
          const uint32_t d = tmem + (uint32_t)((i & 1) * N);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f8f6f4(d, smem_desc_sw128(kaddr + 32 * k, 16, 1024), smem_desc_sw128(qaddr + 32 * k, 16, 1024),
                       idesc_s, k > 0);
          mma_commit(&b.s_full[i & 1]);
        }
        if (i >= 1) {  // O_j^T = V_j^T . P_j^T for the previous tile
          const int j = i - 1, st = j % S;
          ok = mbar_wait(&b.p_full[j & 1], (j >> 1) & 1, abort_flag, MJ_TC_WAIT_NS) &&
               mbar_wait(&b.v_ready[j & 1], (j >> 1) & 1, abort_flag, MJ_TC_WAIT_NS) &&
               mbar_wait(&b.o_free[j & 1], ((j >> 1) & 1) ^ 1, abort_flag, MJ_TC_WAIT_NS);
          if (!ok) break;
          tc_fence_after();
          const uint32_t vaddr = smem_addr(FMT == MJ_KV_E2M3 ? vcvt(j & 1) : vbuf(st));
          const uint32_t paddr = smem_addr(pbuf(j & 1));
          const uint32_t d = tmem + (uint32_t)(2 * N + (j & 1) * N);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_f8f6f4(d, smem_desc_sw128(vaddr + 4096 * k, kTileBytes, 1024),
                       smem_desc_sw128(paddr + 32 * k, 16, 1024), idesc_o, k > 0);
          mma_commit(&b.o_full[j & 1]);
          mma_commit(&b.empty[st]);
          mma_commit(&b.v_free[j & 1]);
        }
      }
      if (!ok && !*abort_flag) give_up();
      // all issued MMAs must complete before TMEM is released
      mma_commit(b.drain);
      mbar_wait(b.drain, 0, &never_abort, MJ_TC_WAIT_NS);
    }
    __syncwarp();
  } else if (warp < kWarpSm0) {
    // ------------------------------------------------ V conversion / tail zero
    const int ct = threadIdx.x - kWarpCvt0 * 32;  // 0..63
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j % S;
      // v_free bounds this role to two tiles ahead of the PV MMA: v_ready is a
      // two-slot barrier pair, and running further ahead would complete a
      // phase the MMA has not waited for yet
      bool ok = mbar_wait(&b.full[st], (j / S) & 1, abort_flag, MJ_TC_WAIT_NS) &&
                mbar_wait(&b.v_free[j & 1], ((j >> 1) & 1) ^ 1, abort_flag, MJ_TC_WAIT_NS);
      if (!ok) {
        if (!*abort_flag) give_up();
        break;
      }
      if (FMT == MJ_KV_E2M3) {
        const uint4* src = reinterpret_cast<const uint4*>(vbuf(st));
        uint4* dst = reinterpret_cast<uint4*>(vcvt(j & 1));
#pragma unroll 4
        for (int c = ct; c < kTileBytes / 16; c += 64) dst[c] = e2m3x16_to_e4m3(src[c]);
        // e2m3 has no NaN code: rows past the sequence end are finite and get P = 0
      } else {
        // e4m3 rows past the sequence end inside its last page may hold NaN
        // bytes; NaN * 0 would poison O, so zero them (their P is 0)
        const int valid = L - (tb + j) * kTileRows;
        if (valid < kTileRows) {
          const int r0 = valid > 0 ? valid : 0;
          uint4* v4 = reinterpret_cast<uint4*>(vbuf(st));
          for (int c = r0 * 8 + ct; c < kTileRows * 8; c += 64) v4[c] = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&b.v_ready[j & 1]);
    }
  } else {
    // --------------------------------------------------- softmax warpgroup
    const int t = threadIdx.x - kWarpSm0 * 32;  // 0..127: TMEM lane = KV row of a tile = head-dim index
    const int wq = warp - kWarpSm0;             // TMEM lane quarter
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const int h_k = a.h_k, h_r = a.h_q / a.h_k, q_len = a.q_len, n_q = q_len * h_r;

    // Q: this thread holds head-dim element t of every query row
    float qv[NQP];
    float qmax = 0.f;
#pragma unroll
    for (int r = 0; r < NQP; ++r) {
      float x = 0.f;
      if (r < n_q) {
        const int qi = r / h_r, rr = r % h_r;
        const int64_t tok = (int64_t)seq * q_len + qi;
        const int qh = h * h_r + rr;
        x = load_elem(a.q, tok * a.q_stride_tok + qh * a.q_stride_head + t, a.q_dtype);
        if (a.q_mul) x *= a.q_mul[(int64_t)qh * 128 + t];
      }
      qv[r] = x;
      qmax = fmaxf(qmax, fabsf(x));
    }
    qmax = warp_max_f32(qmax);
    if (lane == 0) red[wq] = qmax;
    if (t < NQP) lim_s[t] = (t < n_q) ? (a.causal ? L - q_len + t / h_r : L - 1) : -1;
    named_bar_sync(1, 128);
    qmax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    // three-term e4m3 split of q * qs, |q * qs| <= 224
    const float qs = qmax > 0.f ? 224.f / qmax : 1.f;
#pragma unroll
    for (int r = 0; r < NQP; r += 2) {
      uint16_t hb, mb, lb;
      split3(qv[r] * qs, qv[r + 1] * qs, hb, mb, lb);
      store_split<NQP>(qbuf, r, t, hb, mb, lb);
    }
    fence_proxy_async_smem();
    const float kd = descale_at(a.k_descale, a.k_descale_mode, seq, h, h_k);
    const float vd = descale_at(a.v_descale, a.v_descale_mode, seq, h, h_k);
    const float c2 = a.softmax_scale * kd * kLog2e / qs;  // S (in q*qs units) -> log2 units
    named_bar_sync(1, 128);  // all Q bytes written and fenced; red[] reads done
    if (t == 0) mbar_arrive(b.q_full);

    float m[NQP], l[NQP], cr[NQP], oacc[NQP];
#pragma unroll
    for (int r = 0; r < NQP; ++r) {
      m[r] = -INFINITY;
      l[r] = 0.f;
      cr[r] = 1.f;
      oacc[r] = 0.f;
    }
    // fold the O tile of KV tile jj into the register accumulator
    auto fold = [&](int jj) {
      if (!mbar_wait(&b.o_full[jj & 1], (jj >> 1) & 1, abort_flag, MJ_TC_WAIT_NS) && !*abort_flag) give_up();
      tc_fence_after();
      float ov[3 * NQP];
      tmem_ld_cols<NQP>(tmem + (uint32_t)(2 * N + (jj & 1) * N) + lane_base, ov);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&b.o_free[jj & 1]);
#pragma unroll
      for (int r = 0; r < NQP; ++r) oacc[r] = fmaf(oacc[r], cr[r], combine3<NQP>(ov, r));
    };

    bool aborted = false;
    for (int i = 0; i < n_tiles; ++i) {
      if (i >= 1) fold(i - 1);  // uses cr of tile i-1
      if (!mbar_wait(&b.s_full[i & 1], (i >> 1) & 1, abort_flag, MJ_TC_WAIT_NS) && !*abort_flag) give_up();
      tc_fence_after();
      float sv[3 * NQP];
      tmem_ld_cols<NQP>(tmem + (uint32_t)((i & 1) * N) + lane_base, sv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&b.s_free[i & 1]);
      const int j = (tb + i) * kTileRows + t;  // this thread's KV row
      float* rd = red + (i & 1) * 4 * NQP;
#pragma unroll
      for (int r = 0; r < NQP; ++r) {
        float s = combine3<NQP>(sv, r) * c2;
        if (j > lim_s[r]) s = -INFINITY;
        sv[r] = s;
        const float wm = warp_max_f32(s);
        if (lane == 0) rd[wq * NQP + r] = wm;
      }
      // the max exchange barrier doubles as a uniform abort vote
      if (named_bar_or(1, 128, *abort_flag != 0)) {
        aborted = true;
        break;
      }
      unsigned char* pb = pbuf(i & 1);
#pragma unroll
      for (int r = 0; r < NQP; r += 2) {
        float p2[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int rr = r + u;
          const float mt = fmaxf(fmaxf(rd[rr], rd[NQP + rr]), fmaxf(rd[2 * NQP + rr], rd[3 * NQP + rr]));
          const float m_new = fmaxf(m[rr], mt);
          const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
          const float corr = exp2f(m[rr] - m_use);  // m = -inf -> 0
          const float p = exp2f(sv[rr] - m_use);    // masked -> 0
          l[rr] = fmaf(l[rr], corr, p);
          m[rr] = m_new;
          cr[rr] = corr;
          p2[u] = p * kPScale;
        }
        uint16_t hb, mb, lb;
        split3(p2[0], p2[1], hb, mb, lb);
        store_split<NQP>(pb, r, t, hb, mb, lb);
      }
      fence_proxy_async_smem();
      mbar_arrive(&b.p_full[i & 1]);
    }
    if (!aborted) fold(n_tiles - 1);

    // l: per-thread partial sums over this thread's KV rows -> per query row
#pragma unroll
    for (int r = 0; r < NQP; ++r) {
      float x = l[r];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      if (lane == 0) lred[wq * NQP + r] = x;
    }
    aborted = named_bar_or(1, 128, aborted || *abort_flag != 0);
    if (!aborted) {
      const bool final_out = a.n_splits[seq] <= 1;
      const float vscale = (FMT == MJ_KV_E2M3 ? 64.f : 1.f) * vd / kPScale;
      if (!final_out && (split >= a.max_splits || seq >= a.part_seqs || !a.o_part)) {
        if (t == 0) flag(a.status, MJ_DEV_BAD_SPLIT);
      } else {
#pragma unroll
        for (int r = 0; r < NQP; ++r) {
          if (r < n_q) {
            const float lt = lred[r] + lred[NQP + r] + lred[2 * NQP + r] + lred[3 * NQP + r];
            const float inv = lt > 0.f ? vscale / lt : 0.f;
            const int qi = r / h_r, rr = r % h_r;
            const int64_t tok = (int64_t)seq * q_len + qi;
            const int qh = h * h_r + rr;
            float o = oacc[r] * inv;
            const float lse = lt > 0.f ? (m[r] + log2f(lt)) * kLn2 : -INFINITY;
            if (final_out) {
              if (a.o_mul) o *= a.o_mul[(int64_t)qh * 128 + t];
              store_elem(a.o, tok * a.o_stride_tok + qh * a.o_stride_head + t, a.o_dtype, o);
              if (t == 0 && a.lse) a.lse[tok * a.h_q + qh] = lse;
            } else {
              const int64_t row = (((int64_t)split * a.part_seqs + seq) * h_k + h) * n_q + r;
              a.o_part[row * 128 + t] = o;
              if (t == 0) a.lse_part[row] = lse;
            }
          }
        }
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace tc
}  // namespace mj

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
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
  const int n_q = a.q_len * (a.h_q / a.h_k);
  if (a.head_size != 128) return "head_size != 128";
  if (n_q > 16) return "more than 16 query rows per KV head";
  if (a.page_size != 16 && a.page_size != 32 && a.page_size != 64 && a.page_size != 128) return "page size";
  if (a.num_pages >= (int64_t)INT32_MAX) return "num_pages";
  const uintptr_t al = a.kv_format == MJ_KV_E2M3 ? 32 : 16;
  if ((uintptr_t)a.k_cache % al || (uintptr_t)a.v_cache % al) return "KV view alignment";
  const int64_t st[6] = {a.k_stride_page, a.k_stride_row, a.k_stride_head, a.v_stride_page, a.v_stride_row, a.v_stride_head};
  for (int i = 0; i < 6; ++i)
    if (st[i] % (int64_t)al) return "KV stride alignment";
  if (a.k_stride_row == 0 || a.v_stride_row == 0) return "row stride";
  if (!encode_fn()) return "cuTensorMapEncodeTiled unavailable";
  return nullptr;
}

static bool make_map(CUtensorMap* m, const void* base, int64_t s_page, int64_t s_row, int64_t s_head,
                     const mj_decode_args& a) {
  const bool e2m3 = a.kv_format == MJ_KV_E2M3;
  // a dimension of extent 1 never moves its coordinate; give it any legal stride
  const int64_t fill = e2m3 ? 32 : 16;
  cuuint64_t dims[4] = {128, (cuuint64_t)a.page_size, (cuuint64_t)a.h_k, (cuuint64_t)a.num_pages};
  cuuint64_t strides[3] = {(cuuint64_t)(s_row ? s_row : fill), (cuuint64_t)(s_head ? s_head : fill),
                           (cuuint64_t)(s_page ? s_page : fill)};
  cuuint32_t box[4] = {128, (cuuint32_t)a.page_size, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fn()(m, e2m3 ? CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B : CU_TENSOR_MAP_DATA_TYPE_UINT8, 4,
                           const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int FMT, int NQP>
static cudaError_t launch_tc_t(const mj_decode_args& a, const CUtensorMap& mk, const CUtensorMap& mv,
                               cudaStream_t stream) {
  const int smem = tc::Cfg<FMT, NQP>::SMEM;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(tc::decode_tc_kernel<FMT, NQP>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  dim3 grid((unsigned)a.num_work, (unsigned)a.h_k);
  tc::decode_tc_kernel<FMT, NQP><<<grid, tc::kThreads, smem, stream>>>(a, mk, mv);
  return cudaGetLastError();
}

// Launch the tensor-core decode when it can run these arguments; *handled
// tells the caller whether it did. A tensor-map encoding failure is an error.
cudaError_t launch_decode_tc(const mj_decode_args& a, cudaStream_t stream, bool* handled) {
  *handled = false;
  if (tc_ineligible(a)) return cudaSuccess;
  CUtensorMap mk, mv;
  if (!make_map(&mk, a.k_cache, a.k_stride_page, a.k_stride_row, a.k_stride_head, a) ||
      !make_map(&mv, a.v_cache, a.v_stride_page, a.v_stride_row, a.v_stride_head, a))
    return cudaErrorInvalidValue;
  *handled = true;
  const int n_q = a.q_len * (a.h_q / a.h_k);
  if (a.kv_format == MJ_KV_E2M3)
    return n_q <= 8 ? launch_tc_t<MJ_KV_E2M3, 8>(a, mk, mv, stream) : launch_tc_t<MJ_KV_E2M3, 16>(a, mk, mv, stream);
  return n_q <= 8 ? launch_tc_t<MJ_KV_FP8_E4M3, 8>(a, mk, mv, stream) : launch_tc_t<MJ_KV_FP8_E4M3, 16>(a, mk, mv, stream);
}

}  // namespace mj
