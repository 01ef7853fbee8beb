// Paged split-KV decode attention on the 5th-generation tensor cores (sm_100a).
//
// Persistent, warp-specialized CTAs walk a job list: a job is (work item, KV
// head, row group), a work item a contiguous chunk of 128-row KV tiles of one
// sequence (the planner's unit, the reference's arch/thor/plan.py:140-197).
// A job serves RT = NWG x NQP query rows of the KV head (every query head of
// the GQA group and every draft position) from one read of each KV byte.
//
// Data path per 128-row tile:
//   TMA (one box per page through the block table; for the (B, H, N, 2*row)
//   layout one 5-D box lands the page's K and V rows together) -> SMEM ring,
//   128-byte swizzled; e2m3 rows arrive through the 16U6 TMA type (12 packed
//   bytes per 16-byte slot), e4m3 rows as bytes. Pages past the sequence are
//   read at an out-of-range page coordinate: the TMA zero-fills them.
//   S = K . Q^T        tcgen05.mma kind::f8f6f4, M = 128 KV rows, N = 3*RT,
//                      A = K (e4m3 or e2m3, K-major), B = Q split in three
//                      e4m3 terms (row blocks hi, mid = (q - hi) * 16,
//                      lo = (q - hi - mid/16) * 256, RT rows each)
//   softmax            NWG warpgroups, thread = TMEM lane = KV row; base-2
//                      online softmax in fp32 with a lazily raised max; P
//                      split into three e4m3 terms (scaled by 448/256),
//                      stored MN-major for the next MMA
//   O^T += V^T . P^T   tcgen05.mma kind::f8f6f4, M = 128 head-dim rows,
//                      A = V (e4m3, MN-major), B = P; O accumulates in TMEM
//                      over the job's tiles and is rescaled in place on the
//                      rare max raise, read out once at the job's end
//   e2m3 V cannot be an MN-major MMA operand, so converter warps (a whole
//   warpgroup in the one-warpgroup variants) rewrite each 16-code slot in
//   place as 16 e4m3 bytes of value code * 2^-6 (exact; the 2^6 is folded
//   into the output scale); e3m2 and e2m1 likewise. nvfp4 (e2m1 codes with an
//   e4m3 scale per 16) converts K and V: each slot becomes
//   e4m3(code * scale * 2^-3), its scale rows arriving with the stage.
//
// Numerics: split-fp8 Q and P carry ~12 significant bits each (hi + mid /
// 16 + lo / 256 of the fp32 value), accumulation is fp32 in TMEM, the
// softmax is fp32;
// the reference's single-e4m3 recipe (arch/thor/decode.py:1288-1297) is not
// used because it misses the 2e-3 tolerance.
//
// Every mbarrier wait is bounded (MJ_TC_WAIT_NS); on a timeout the CTA sets
// MJ_DEV_TIMEOUT in the status word, all roles stop at their next wait, wait
// (bounded) for their in-flight copies and MMAs, free TMEM and return.
// mj_decode_args.abort_probe_ns makes the S issuer start with a wait that
// runs out, to exercise that path.
#pragma once

#include <limits.h>
#include <math.h>

#include <atomic>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

#ifndef MJ_D256_SMV
#define MJ_D256_SMV 1
#endif
#ifndef MJ_D256_SM_CHUNKS
#define MJ_D256_SM_CHUNKS 512
#endif
#ifndef MJ_NVFP4_SMV
#define MJ_NVFP4_SMV 1
#endif
#ifndef MJ_CVT_BALANCED
#define MJ_CVT_BALANCED 1
#endif
#ifndef MJ_TC_WAIT_NS
#define MJ_TC_WAIT_NS 500000000ull  // 0.5 s per wait: a tile takes microseconds
#endif

namespace mj {
namespace tc {

using namespace sm100;

constexpr int kTileBytes = 128 * 128;  // one 128 x 128 byte operand tile (e2m3: 16U6 slots)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
// The running max m is raised only when a score exceeds it by more than
// kRescaleLog2 (log2 units; the rest of the time no cross-thread max is
// needed), so p = 2^(s - m) <= 2^8. The softmax keeps m' = m - log2(448/256)
// instead of m, so 2^(s - m') = p * 448/256 <= 448 fits e4m3 as written, the
// row sums carry the same factor (it cancels in O = sum(p' v) / sum(p')), and
// the LSE is m' + log2(sum p') unchanged.
constexpr float kRescaleLog2 = 8.0f;
constexpr float kLog2PScale = 0.80735492205760410f;  // log2(448 / 256)
// the in-kernel split merge holds one partial per split in registers
constexpr int kMergeMaxSplits = 16;

// warp roles of the first warpgroup: TMA producer, the S MMA issuer, a
// converter warp and the PV MMA issuer (two issuers, each blocking on its
// own barriers: neither waits behind the other's inputs)
constexpr int kWarpTma = 0;
constexpr int kWarpMma = 1;
constexpr int kWarpCvt = 2;
constexpr int kWarpPv = 3;
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

// e3m2: the same spread, then the 5 magnitude bits move up one place (e4m3
// keeps the 3-bit exponent over bias 7 and gains a mantissa bit): value * 2^-4.
__device__ __forceinline__ uint32_t e3m2_bytes(uint32_t t) { return ((t & 0x1F1F1F1Fu) << 1) | (t & 0x80808080u); }
__device__ __forceinline__ uint4 e3m2x16_to_e4m3(uint4 raw) {
  const uint4 t = e2m3x16_to_e4m3(raw);
  return make_uint4(e3m2_bytes(t.x), e3m2_bytes(t.y), e3m2_bytes(t.z), e3m2_bytes(t.w));
}

// e2m1: a 16U4 slot holds 16 nibbles in its first 8 bytes; code s|e|m becomes
// byte s<<7 | e<<3 | m<<2, value * 2^-6 (subnormals included). The even
// codes (low nibbles) and the odd ones (high nibbles) of a word become e4m3
// bytes where they sit, then one byte permute per output word interleaves
// them.
__device__ __forceinline__ uint32_t e2m1_even_bytes(uint32_t w) {
  return ((w & 0x07070707u) << 2) | ((w & 0x08080808u) << 4);
}
__device__ __forceinline__ uint32_t e2m1_odd_bytes(uint32_t w) {
  return ((w >> 2) & 0x1C1C1C1Cu) | (w & 0x80808080u);
}
__device__ __forceinline__ uint4 e2m1x16_to_e4m3(uint4 raw) {
  const uint32_t e0 = e2m1_even_bytes(raw.x), o0 = e2m1_odd_bytes(raw.x);
  const uint32_t e1 = e2m1_even_bytes(raw.y), o1 = e2m1_odd_bytes(raw.y);
  return make_uint4(__byte_perm(e0, o0, 0x5140), __byte_perm(e0, o0, 0x7362), __byte_perm(e1, o1, 0x5140),
                    __byte_perm(e1, o1, 0x7362));
}

// nvfp4: 8 e2m1 codes (nibbles of w, code 0 lowest) -> 8 e4m3 bytes
// e4m3(value(code) * scale * 2^-3), given t = the 8 bytes e4m3(value(m) *
// scale * 2^-3) of the group's scale for magnitudes m = 0..7 (built once per
// CTA for every scale byte). The magnitude bytes come from one byte permute
// per 4 codes; the signs from a permute in sign-replicate mode (a selector
// nibble with bit 3 set copies the msb of the chosen byte over the output
// byte): code 2i's sign is the msb of byte i of w << 4, code 2i+1's of byte i
// of w. e4m3 rounding is symmetric in the sign, so this is the same byte.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint2 nvfp4x8_to_e4m3(uint32_t w, uint2 t) {
  const uint32_t mag_lo = prmt(t.x, t.y, w & 0x7777u);
  const uint32_t mag_hi = prmt(t.x, t.y, (w >> 16) & 0x7777u);
  const uint32_t a = w << 4;
  const uint32_t sg_lo = prmt(a, w, 0xD9C8u);  // msb of a.b0, w.b0, a.b1, w.b1
  const uint32_t sg_hi = prmt(a, w, 0xFBEAu);  // msb of a.b2, w.b2, a.b3, w.b3
  return make_uint2(mag_lo | (sg_lo & 0x80808080u), mag_hi | (sg_hi & 0x80808080u));
}

// Per-format constants of the tensor-core path.
template <int FMT>
struct Fmt {
  static constexpr bool NARROW = FMT != MJ_KV_FP8_E4M3;  // V needs a conversion to e4m3
  static constexpr bool SCALED = FMT == MJ_KV_NVFP4;     // group scales: K is converted too
  // kind::f8f6f4 operand format of K (nvfp4 K is converted to e4m3)
  static constexpr uint32_t MMA_FMT = FMT == MJ_KV_E2M3 ? 3u : FMT == MJ_KV_E3M2 ? 4u : FMT == MJ_KV_E2M1 ? 5u : 0u;
  static constexpr uint32_t ROW = (FMT == MJ_KV_E2M1 || SCALED) ? 64u : NARROW ? 96u : 128u;  // packed bytes per 128-code row
  static constexpr float V_UNSCALE = FMT == MJ_KV_E3M2 ? 16.f : SCALED ? 1.f : NARROW ? 64.f : 1.f;  // undoes the conversion's shift
  static __device__ __forceinline__ uint4 convert(uint4 raw) {
    if constexpr (FMT == MJ_KV_E3M2) return e3m2x16_to_e4m3(raw);
    else if constexpr (FMT == MJ_KV_E2M1) return e2m1x16_to_e4m3(raw);
    else return e2m3x16_to_e4m3(raw);
  }
};

// warp 2 (and, with CVTW, a whole second warpgroup): V conversion (e2m3) /
// tail zeroing (e4m3); then NWG softmax warpgroups of 4 warps

// A CTA runs NWG softmax warpgroups of NQP query rows each (RT = NWG * NQP
// rows per job). One warpgroup: two CTAs per SM; several: one CTA per SM that
// streams each KV tile once for all its rows. CVTW = 1 adds a warpgroup of
// converter warps so that the softmax warpgroup converts no V. DH = 2 runs
// head_dim 256 as two 128-wide halves: each stage holds both halves of K and
// V, S sums 8 K-steps, O is two TMEM blocks (one per half), each softmax
// thread owns head-dim elements t and 128 + t; one CTA per SM.
template <int FMT, int NQP, int NWG, int CVTW, int DH = 1>
struct Cfg {
  static_assert(DH == 1 || (DH == 2 && NWG == 1), "head_dim 256: one warpgroup");
  static constexpr int RT = NWG * NQP;
  static constexpr int SM0 = 4 * (1 + CVTW);             // first softmax warp
  static constexpr int THREADS = 128 * (1 + CVTW + NWG);
  static constexpr int CTAS_PER_SM = NWG == 1 && DH == 1 ? 2 : 1;
  // threads of the converter role: warp 2, or (MJ_CVT_BALANCED) with a
  // converter warpgroup that warpgroup alone, one converter warp per SM
  // sub-partition beside each softmax warp
  static constexpr int CVT_ROLE = (MJ_CVT_BALANCED && CVTW) ? 128 : 32 + 128 * CVTW;
  static constexpr int CVT_BASE = (MJ_CVT_BALANCED && CVTW) ? 0 : 32;  // converter index of the warpgroup's thread 0
  static constexpr bool SM_CONVERTS = Fmt<FMT>::NARROW && CVTW == 0;  // softmax warpgroups share the conversion
  static constexpr int CVT_THREADS = CVT_ROLE + (SM_CONVERTS ? 128 * NWG : 0);  // threads that convert a V tile
  // nvfp4 at 4 rows per KV head: the converter warpgroup converts K (on the
  // S MMA's path), the softmax warpgroup converts V after publishing P (ns
  // shape +5 %; at 8 rows the softmax has no room for it: -10 %)
  static constexpr bool SM_CVT_V = MJ_NVFP4_SMV && Fmt<FMT>::SCALED && NWG == 1 && NQP <= 4 && DH == 1;
  // head_dim 256, narrow formats: the softmax warpgroup converts part of the
  // V tile after publishing P, the converter warpgroup the rest
  static constexpr bool SM_CVT_VHI = MJ_D256_SMV && DH == 2 && Fmt<FMT>::NARROW && !Fmt<FMT>::SCALED;
  // of the 2 x 1024 16-byte chunks of such a V tile: the last SM_CHUNKS to the
  // softmax warpgroup, the others to the converter warpgroup (at the
  // reference's head shape, e2m3: none 0.186 ms, 1024 0.181, 512 0.168, 256 0.174)
  static constexpr int SM_CHUNKS = SM_CVT_VHI ? MJ_D256_SM_CHUNKS : 0;
  // Query rows enter the MMAs as three row blocks (hi, mid, lo) of RT rows;
  // warpgroup w owns rows w * NQP .. of each block.
  static constexpr int NS = (3 * RT + 7) / 8 * 8 < 16 ? 16 : (3 * RT + 7) / 8 * 8;  // S MMA N (Q is K-major)
  static constexpr int NO = (3 * RT + 15) / 16 * 16;     // PV MMA N (P is MN-major: multiples of 16)
  static constexpr int QBYTES = NS * 128;                // one K-major Q operand
  static constexpr int PBYTES = NO * 128;                // one MN-major P operand: NO/16 groups of [128 s][16 B]
  // (nvfp4 at 8 rows: its scale copies leave room for two stages at two CTAs per SM)
  static constexpr int STAGES = DH == 2 ? (NQP <= 8 && !Fmt<FMT>::SCALED ? 3 : 2)
                               : NWG == 1 ? (NQP <= 4 || (NQP == 8 && !Fmt<FMT>::SCALED) ? 3 : 2) : NWG == 2 ? 5 : 4;
  static_assert(DH == 1 || !SM_CONVERTS, "head_dim 256: narrow formats convert on a converter warpgroup");
  static_assert(!Fmt<FMT>::SCALED || CVTW == 1, "nvfp4 converts K on the converter warpgroup only");
  static constexpr int TCOLS = 2 * NS + DH * NO;         // S0 S1 O (O accumulates over a job's tiles; DH blocks)
  static constexpr int TMEM_COLS = TCOLS <= 32 ? 32 : TCOLS <= 64 ? 64 : TCOLS <= 128 ? 128 : TCOLS <= 256 ? 256 : 512;
  static_assert(TCOLS * CTAS_PER_SM <= 512, "the CTAs of an SM share its 512 TMEM columns");
  static_assert(NWG == 1 || NQP % 16 == 0, "several warpgroups write whole 16-row P groups");
  // Register split (setmaxnreg) when the launch allocation is too tight for
  // the softmax rows (512 threads at one CTA per SM: 128 each; 384 threads at
  // two: 80): the TMA / MMA / converter warpgroups keep REG_LO, the softmax
  // ones get REG_HI. REG_POOL must fit THREADS x the launch registers (checked
  // on the host before the first launch).
  static constexpr int REG_LO = DH == 2 ? 0 : NWG == 3 ? (CVTW ? 48 : 64) : CVTW ? 56 : 0;
  static constexpr int REG_HI = DH == 2 ? 0 : NWG == 3 ? (CVTW ? 128 : 144) : CVTW ? 128 : 0;
  static constexpr int REG_POOL = 128 * REG_LO * (1 + CVTW) + 128 * NWG * REG_HI;
  static constexpr uint32_t K_TX = 128u * Fmt<FMT>::ROW;  // bytes TMA reads per tile operand
  // shared memory plan (offsets from the 1024-aligned dynamic shared memory base)
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + STAGES * DH * kTileBytes;
  static constexpr int Q_OFF = V_OFF + STAGES * DH * kTileBytes;  // two slots (jobs) x DH halves
  static constexpr int P_OFF = (Q_OFF + 2 * DH * QBYTES + 1023) / 1024 * 1024;  // two slots (tiles)
  static constexpr int BAR_OFF = P_OFF + 2 * PBYTES;
  static constexpr int NBARS = 5 * STAGES + 2 * 8 + 2;  // k/v full/empty rings, k_ready ring, 8 pairs, drain, never
  // float red[NWG][2][4][NQP], 16-byte aligned so its rows load as float4
  static constexpr int RED_OFF = (BAR_OFF + NBARS * 8 + 15) / 16 * 16;
  static constexpr int MISC_OFF = RED_OFF + NWG * 2 * 4 * NQP * 4;  // tmem base, abort, never_abort, l scratch [NWG][4][NQP]
  // nvfp4: per stage the K then V scale rows of the tile ([128 rows][8 B] each)
  static constexpr int SC_OFF = (MISC_OFF + 64 + NWG * 4 * 4 * NQP + 15) / 16 * 16;
  static constexpr int SC_BYTES = Fmt<FMT>::SCALED ? STAGES * DH * 2 * 128 * 8 : 0;  // per half: 8 B a row
  // nvfp4: for each of the 256 scale bytes the e4m3 bytes of the 8 code magnitudes
  static constexpr int LUT_OFF = SC_OFF + SC_BYTES;
  static constexpr int SMEM = LUT_OFF + (Fmt<FMT>::SCALED ? 256 * 8 : 0);
};

struct Bars {
  uint64_t *k_full, *k_empty, *v_full, *v_empty;               // TMA rings
  uint64_t* k_ready;                                          // nvfp4: K tile converted (ring)
  uint64_t *s_full, *s_free, *p_full, *o_full, *v_ready, *v_free, *q_full;  // pairs (o_full: PV of tile t done)
  uint64_t* o_free;                                         // once per job: O read out, next job may overwrite
  uint64_t* drain;
};


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

// Stores the three-term split of rows r, r+1 (column t) into a K-major tile
// whose hi / mid / lo row blocks are RT rows each.
template <int RT>
__device__ __forceinline__ void store_split(unsigned char* buf, int r, int t, uint16_t hb, uint16_t mb, uint16_t lb) {
  buf[sw128_offset(r, t)] = (uint8_t)(hb & 0xFF);
  buf[sw128_offset(r + 1, t)] = (uint8_t)(hb >> 8);
  buf[sw128_offset(RT + r, t)] = (uint8_t)(mb & 0xFF);
  buf[sw128_offset(RT + r + 1, t)] = (uint8_t)(mb >> 8);
  buf[sw128_offset(2 * RT + r, t)] = (uint8_t)(lb & 0xFF);
  buf[sw128_offset(2 * RT + r + 1, t)] = (uint8_t)(lb >> 8);
}

// C TMEM columns (a multiple of 8) of this thread's lane -> v
template <int C>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, float* v) {
#pragma unroll
  for (int c = 0; c + 16 <= C; c += 16) tmem_ld16(taddr + c, v + c);
  if (C % 16) tmem_ld8(taddr + (C / 16) * 16, v + (C / 16) * 16);
}

// rows r, r+1 of the three row blocks: hi + mid / 16 + lo / 256
template <int NQP>
__device__ __forceinline__ float2 combine3x2(const float* v, int r) {
  const float2 hi = make_float2(v[r], v[r + 1]), mid = make_float2(v[NQP + r], v[NQP + r + 1]),
               lo = make_float2(v[2 * NQP + r], v[2 * NQP + r + 1]);
  return ffma2(lo, make_float2(0.00390625f, 0.00390625f), ffma2(mid, make_float2(0.0625f, 0.0625f), hi));
}

// split3 on a pair with packed residual arithmetic (the residuals are exact):
// y = hi + mid / 16 + lo / 256, each term e4m3. Used for P (0 <= y <= 448).
// A variant that first rounds y to f16 (three fewer instructions a pair)
// measured 4x the output error at the config-3 shape (0.0026 max-abs against
// the oracle where |o| reaches 13, beyond the 2e-3 tolerance); this one
// stays at 7e-4.
__device__ __forceinline__ void split3x2(float2 y, uint16_t& hb, uint16_t& mb, uint16_t& lb) {
  const float2 m16 = make_float2(-16.f, -16.f), p16 = make_float2(16.f, 16.f);
  hb = f2_to_e4m3x2(y.x, y.y);
  const float2 r1 = ffma2(e4m3x2_to_f2(hb), m16, fmul2(y, p16));
  mb = f2_to_e4m3x2(r1.x, r1.y);
  const float2 r2 = ffma2(e4m3x2_to_f2(mb), m16, fmul2(r1, p16));
  lb = f2_to_e4m3x2(r2.x, r2.y);
}


}  // namespace tc
}  // namespace mj

namespace mj {
namespace tc {

// FUSED: K and V of a page arrive in one TMA box (the vLLM / reference layout
// (pages, h_k, page_size, K row | V row)); the box lands as alternating 1 KB
// K and V swizzle atoms, so both operands see an atom stride of 2048 B.
// Otherwise K and V are separate boxes into separate tiles (atom stride 1024 B).
// Head_dim 256 (DH = 2): every box is one 128-code half of the rows (fused:
// tmk maps half 0, tmv half 1; otherwise a halves dimension in each map).
template <int FMT, int NQP, int NWG, int CVTW, bool FUSED, int DH>
__global__ void __launch_bounds__(Cfg<FMT, NQP, NWG, CVTW, DH>::THREADS, Cfg<FMT, NQP, NWG, CVTW, DH>::CTAS_PER_SM)
    decode_tc_kernel(const __grid_constant__ mj_decode_args a, const __grid_constant__ CUtensorMap tmk,
                     const __grid_constant__ CUtensorMap tmv) {
  using C = Cfg<FMT, NQP, NWG, CVTW, DH>;
  constexpr int D = 128 * DH;  // head_dim
  constexpr int NS = C::NS, NO = C::NO, RT = C::RT;
  constexpr int S = C::STAGES;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* sm = smem_raw;  // 1024-aligned: the 128-byte swizzle atoms need it
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (reinterpret_cast<uintptr_t>(sm) & 1023) {  // uniform: no barrier or TMEM touched yet
    if (threadIdx.x == 0) flag(a.status, MJ_DEV_BAD_SPLIT);
    return;
  }
  const int h_k = a.h_k;
  // the limit of every pipeline wait (drains keep the default: copies and
  // MMAs in flight must land before the CTA exits, however short this is)
  // every pipeline wait is bounded by MJ_TC_WAIT_NS (a compile-time limit:
  // a run-time one on every wait measured 1-3 % slower)
  constexpr uint64_t wait_ns = MJ_TC_WAIT_NS;
  // A job is (work item, KV head, row group): a CTA serves at most RT query
  // rows; a larger GQA x draft group is cut into n_rg row groups whose jobs
  // are adjacent in the list, so CTAs reading the same KV stream run side by
  // side and the repeat reads hit L2.
  const int n_q_all = a.q_len * (a.h_q / h_k);
  const int n_rg = (n_q_all + RT - 1) / RT;
  const int total_jobs = a.num_work * h_k * n_rg;

  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  Bars b;
  b.k_full = bars;
  b.k_empty = bars + S;
  b.v_full = bars + 2 * S;
  b.v_empty = bars + 3 * S;
  b.s_full = bars + 4 * S;
  b.s_free = b.s_full + 2;
  b.p_full = b.s_free + 2;
  b.o_full = b.p_full + 2;
  b.o_free = b.o_full + 2;
  b.v_ready = b.o_free + 2;
  b.v_free = b.v_ready + 2;
  b.q_full = b.v_free + 2;
  b.drain = b.q_full + 2;
  b.k_ready = b.drain + 1;
  float* red_all = reinterpret_cast<float*>(sm + C::RED_OFF);   // [NWG][2][4][NQP]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + C::MISC_OFF);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + C::MISC_OFF + 4);
  int& never_abort = *reinterpret_cast<int*>(sm + C::MISC_OFF + 8);  // no one sets it: drains wait on time only
  float* lred_all = reinterpret_cast<float*>(sm + C::MISC_OFF + 64);  // [NWG][4][NQP]

  if (threadIdx.x == 0) {
    // nvfp4: the 32 TMA-warp lanes' scale copies also arrive on the full barriers
    constexpr int FULL = 1 + (Fmt<FMT>::SCALED ? 32 : 0);
    for (int i = 0; i < S; ++i) {
      mbar_init(&b.k_full[i], FULL);
      mbar_init(&b.k_empty[i], 1);
      mbar_init(&b.v_full[i], FULL);
      mbar_init(&b.v_empty[i], 1);  // released by the PV MMA
      mbar_init(&b.k_ready[i], C::CVT_ROLE);  // nvfp4: every converter thread converts K, then V
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b.s_full[i], 1);
      mbar_init(&b.s_free[i], 128 * NWG);
      mbar_init(&b.p_full[i], 128 * NWG);
      mbar_init(&b.o_full[i], 1);
      if (i == 0) mbar_init(b.o_free, 128 * NWG);
      // narrow formats: the converter role (and, without a converter
      // warpgroup, the softmax warpgroups) share the V conversion
      mbar_init(&b.v_ready[i], C::SM_CVT_V ? 128 : Fmt<FMT>::NARROW ? C::CVT_THREADS + (C::SM_CVT_VHI ? 128 : 0) : C::CVT_ROLE);
      mbar_init(&b.v_free[i], 1);
      mbar_init(&b.q_full[i], NWG);
    }
    mbar_init(b.drain, 2);  // one commit from each MMA issuer
    mbar_init(b.k_ready + S, 1);  // "never": nothing arrives on it (the abort-path probe)
    *abort_flag = 0;
    never_abort = 0;
    fence_mbar_init();
  }
  if constexpr (Fmt<FMT>::SCALED) {
    // e4m3(value(m) * scale * 2^-3) for every scale byte and magnitude m
    // (quant.py:81-83: an exact fp32 product, one rounding); a NaN scale byte,
    // which the quantizer never writes, gives zeros
    uint2* lut = reinterpret_cast<uint2*>(sm + C::LUT_OFF);
    for (int e = threadIdx.x; e < 256; e += blockDim.x) {
      uint32_t lo = 0, hi = 0;
      if ((e & 0x7F) != 0x7F) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          lo |= (uint32_t)nvfp4_byte((uint32_t)m, (uint8_t)e) << (8 * m);
          hi |= (uint32_t)nvfp4_byte((uint32_t)(m + 4), (uint8_t)e) << (8 * m);
        }
      }
      lut[e] = make_uint2(lo, hi);
    }
  }
  if (warp == kWarpTma && lane == 0) {
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  // PDL: wait for the cache write before it before any global read, and
  // before taking TMEM, so a waiting CTA holds no tensor memory.
  griddep_wait();
  if (warp == kWarpMma) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S0 [0,NS) S1 [NS,2NS) O [2NS,2NS+NO)
  // Every CTA is resident and holds its TMEM: the combine launch behind this
  // grid (no TMEM, no shared memory) may be scheduled and wait on the GPU.
  if (a.with_combine) griddep_launch_dependents();

  constexpr uint32_t ATOM = FUSED ? 2048u : 1024u;  // byte stride between 8-row swizzle atoms of K (or V)
  auto kbuf = [&](int st, int dh = 0) {
    return FUSED ? sm + (st * DH + dh) * 2 * kTileBytes : sm + C::K_OFF + (st * DH + dh) * kTileBytes;
  };
  auto vbuf = [&](int st, int dh = 0) {
    return FUSED ? sm + (st * DH + dh) * 2 * kTileBytes + 1024 : sm + C::V_OFF + (st * DH + dh) * kTileBytes;
  };
  // byte offset of 16-byte chunk c (row c / 8) of the V tile, and of row r
  auto vchunk = [&](int c) { return (uint32_t)((c >> 6) * ATOM + (c & 63) * 16); };
  auto qbuf = [&](int i, int dh = 0) { return sm + C::Q_OFF + (i * DH + dh) * C::QBYTES; };
  // nvfp4 K / V scale rows of a stage (and head-dim half): [128 rows][8 B]
  auto kscl = [&](int st, int dh = 0) { return sm + C::SC_OFF + (st * DH + dh) * 2048; };
  auto vscl = [&](int st, int dh = 0) { return sm + C::SC_OFF + (st * DH + dh) * 2048 + 1024; };
  auto pbuf = [&](int i) { return sm + C::P_OFF + i * C::PBYTES; };
  auto give_up = [&]() {
    *abort_flag = 1;
    flag(a.status, MJ_DEV_TIMEOUT);
  };
  // every role walks the same job list and skips the same empty items
  auto job = [&](int p, int& seq, int& tb, int& te, int& split, int& h, int& g) {
    g = p % n_rg;
    p /= n_rg;
    const int4 wi = reinterpret_cast<const int4*>(a.work)[p / h_k];
    seq = wi.x;
    tb = wi.y;
    te = wi.z;
    split = wi.w;
    h = p % h_k;
    return te > tb;
  };

  // nvfp4: convert a K or V tile in place (thread ct of the converter role
  // takes chunks ct, ct + CVT_ROLE, ...): the 16 codes of a 16U4 slot are one
  // scale group, whose logical index within the row is the slot's swizzled
  // position XOR the row (mod 8); rows at or past `valid` become zeros.
  auto nvfp4_tile = [&](unsigned char* buf, const unsigned char* scl, int valid, int ct, int nthr) {
    const uint2* lut = reinterpret_cast<const uint2*>(sm + C::LUT_OFF);
#pragma unroll 2
    for (int c = ct; c < kTileBytes / 16; c += nthr) {
      const int r = c >> 3;
      uint4* q = reinterpret_cast<uint4*>(buf + vchunk(c));
      if (r < valid) {
        const uint2 t = lut[scl[r * 8 + ((c ^ r) & 7)]];
        const uint4 raw = *q;
        const uint2 o0 = nvfp4x8_to_e4m3(raw.x, t), o1 = nvfp4x8_to_e4m3(raw.y, t);
        *q = make_uint4(o0.x, o0.y, o1.x, o1.y);
      } else {
        *q = make_uint4(0, 0, 0, 0);
      }
    }
  };

  // ---------------------------------------- V conversion / tail zero (thread ct)
  auto convert_role = [&](const int ct) {
    int it = 0;
    bool ok = true;
    for (int p = blockIdx.x; ok && p < total_jobs; p += gridDim.x) {
      int seq, tb, te, split, h, g;
      if (!job(p, seq, tb, te, split, h, g)) continue;
      const int L = a.seq_lens[seq];
      for (int tile = tb; tile < te; ++tile, ++it) {
        const int st = it % S;
        if constexpr (Fmt<FMT>::SCALED) {
          // every converter thread converts its share of K (which the S MMA
          // waits for) and then of V (needed only by the PV MMA; v_free keeps
          // this role at most two tiles ahead of it)
          const int valid = L - tile * kTileRows;
          ok = mbar_wait(&b.k_full[st], (it / S) & 1, abort_flag, wait_ns);
          if (!ok) break;
#pragma unroll
          for (int dh = 0; dh < DH; ++dh) nvfp4_tile(kbuf(st, dh), kscl(st, dh), valid, ct, C::CVT_ROLE);
          fence_proxy_async_smem();
          mbar_arrive(&b.k_ready[st]);
          if constexpr (C::SM_CVT_V) continue;
          ok = (FUSED || mbar_wait(&b.v_full[st], (it / S) & 1, abort_flag, wait_ns)) &&
               mbar_wait(&b.v_free[it & 1], ((it >> 1) & 1) ^ 1, abort_flag, wait_ns);
          if (!ok) break;
#pragma unroll
          for (int dh = 0; dh < DH; ++dh) nvfp4_tile(vbuf(st, dh), vscl(st, dh), valid, ct, C::CVT_ROLE);
          fence_proxy_async_smem();
          mbar_arrive(&b.v_ready[it & 1]);
          continue;
        }
        // v_free keeps this role at most two tiles ahead of the PV MMA (v_ready is a pair)
        ok = mbar_wait(FUSED ? &b.k_full[st] : &b.v_full[st], (it / S) & 1, abort_flag, wait_ns) &&
             mbar_wait(&b.v_free[it & 1], ((it >> 1) & 1) ^ 1, abort_flag, wait_ns);
        if (!ok) break;
        if constexpr (Fmt<FMT>::NARROW) {
          // in place: the 16 e4m3 bytes of a 16-code group take its 16-byte slot;
          // this role converts chunks ct, ct + CVT_THREADS, ...; without a
          // converter warpgroup the softmax warpgroups convert the others
          // after publishing P
          if constexpr (C::SM_CVT_VHI) {  // chunk g of the tile: half g / 1024, chunk g % 1024
#pragma unroll 2
            for (int g = ct; g < DH * (kTileBytes / 16) - C::SM_CHUNKS; g += C::CVT_THREADS) {
              uint4* q = reinterpret_cast<uint4*>(vbuf(st, g >> 10) + vchunk(g & 1023));
              *q = Fmt<FMT>::convert(*q);
            }
          } else {
#pragma unroll
            for (int dh = 0; dh < DH; ++dh) {
              unsigned char* vb = vbuf(st, dh);
#pragma unroll 2
              for (int c = ct; c < kTileBytes / 16; c += C::CVT_THREADS) {
                uint4* q = reinterpret_cast<uint4*>(vb + vchunk(c));
                *q = Fmt<FMT>::convert(*q);
              }
            }
          }
          // narrow formats have no NaN code: rows past the sequence end are finite and get P = 0
        } else {
          // e4m3 rows past the sequence end inside its last page may hold NaN
          // bytes; NaN * 0 would poison O, so zero them (their P is 0)
          const int valid = L - tile * kTileRows;
          if (valid < kTileRows) {
            const int r0 = valid > 0 ? valid : 0;
            for (int dh = 0; dh < DH; ++dh) {
              unsigned char* vb = vbuf(st, dh);
              for (int c = r0 * 8 + ct; c < kTileRows * 8; c += C::CVT_ROLE)
                *reinterpret_cast<uint4*>(vb + vchunk(c)) = make_uint4(0, 0, 0, 0);
            }
          }
        }
        fence_proxy_async_smem();
        mbar_arrive(&b.v_ready[it & 1]);
      }
    }
    if (!ok && !*abort_flag) give_up();
  };

  if (warp < 4) {
    // the TMA / MMA / converter warpgroup
    if constexpr (C::REG_LO > 0) setmaxnreg_dec<C::REG_LO>();
    if (warp == kWarpTma) {
      // ---------------------------------------------------------------- producer
      const int PS = a.page_size;
      const int P = kTileRows / PS;  // pages per tile; lane p < P loads page p
      // a KV stream read by one job is evicted first; row groups of one KV
      // head re-read it from L2, so their loads keep the normal policy
      const uint64_t kv_policy = n_rg > 1 ? l2_policy_evict_normal() : l2_policy_evict_first();
      int it = 0, k_issued = 0, v_issued = 0;
      bool ok = true;
      for (int p = blockIdx.x; ok && p < total_jobs; p += gridDim.x) {
        int seq, tb, te, split, h, g;
        if (!job(p, seq, tb, te, split, h, g)) continue;
        const int L = a.seq_lens[seq];
        const int32_t* bt = a.block_table + (int64_t)seq * a.block_table_stride;
        // A tile's block-table entries (lane p < P: page p; INT_MIN past the
        // sequence) are loaded while the tile before it is issued and checked
        // only when their own tile is, so the table's memory round trip --
        // long while HBM is saturated -- overlaps the stage wait instead of
        // stalling every issue. Loading further ahead measured slower: issuing
        // faster than the stages turn over raises the memory latency without
        // adding bandwidth.
        auto page_load = [&](int tile) -> int {
          const int row0 = tile * kTileRows + lane * PS;
          return (tile < te && lane < P && row0 < L) ? __ldg(bt + row0 / PS) : INT_MIN;
        };
        auto page_check = [&](int v) -> int {
          if (v == INT_MIN) return (int)a.num_pages;  // out of range -> the TMA zero-fills the box
          if (v < 0 || (int64_t)v >= a.num_pages) {
            flag(a.status, MJ_DEV_BAD_PAGE);  // never dereferenced: zero-filled like a page past the end
            return (int)a.num_pages;
          }
          return v;
        };
        // nvfp4: the 8-byte scale rows of this tile's valid rows (rows lane +
        // 32 i), K or V, into the stage (rows past the sequence are left
        // stale: the converter zeroes those rows); each lane then arrives once
        // per full barrier, when its copies have landed
        auto copy_scales = [&](int tile, int pg, int st, bool v) {
          const int valid = L - tile * kTileRows;
          const unsigned char* base = reinterpret_cast<const unsigned char*>(v ? a.v_scales : a.k_scales);
          const int64_t sp = v ? a.vs_stride_page : a.ks_stride_page, sr = v ? a.vs_stride_row : a.ks_stride_row;
          const int64_t sh = v ? a.vs_stride_head : a.ks_stride_head;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = lane + 32 * i;
            const int pr = __shfl_sync(0xffffffffu, pg, r / PS);
            if (r < valid && pr < a.num_pages) {
              const unsigned char* src = base + (int64_t)pr * sp + (int64_t)(r % PS) * sr + (int64_t)h * sh;
#pragma unroll
              for (int dh = 0; dh < DH; ++dh)  // head_dim 256: 16 scale bytes a row, 8 per half
                cp_async8((v ? vscl(st, dh) : kscl(st, dh)) + r * 8, src + dh * 8);
            }
          }
        };
        // one tile into stage it % S once the stage is free; false on give-up
        auto issue_tile = [&](int tile, int pg) -> bool {
          const int st = it % S;
          const uint32_t par = ((it / S) & 1) ^ 1;
          bool go = true;
          if (FUSED) {  // one box per page: K and V rows together (the stage frees after PV)
            if (lane == 0) go = mbar_wait(&b.v_empty[st], par, abort_flag, wait_ns);
            if (!__shfl_sync(0xffffffffu, go, 0)) return false;
            if (lane == 0) mbar_arrive_expect_tx(&b.k_full[st], 2 * DH * C::K_TX);
            __syncwarp();
            if (lane < P) {
#pragma unroll
              for (int dh = 0; dh < DH; ++dh)
                tma_load_5d(kbuf(st, dh) + lane * PS * 256, dh ? &tmv : &tmk, &b.k_full[st], 0, 0, 0, 0, pg * h_k + h,
                            kv_policy);
            }
            if constexpr (Fmt<FMT>::SCALED) {
              copy_scales(tile, pg, st, false);
              copy_scales(tile, pg, st, true);
              cp_async_arrive_noinc(&b.k_full[st]);
            }
            k_issued = ++it;
            return true;
          }
          if (lane == 0) go = mbar_wait(&b.k_empty[st], par, abort_flag, wait_ns);
          if (!__shfl_sync(0xffffffffu, go, 0)) return false;
          if (lane == 0) mbar_arrive_expect_tx(&b.k_full[st], DH * C::K_TX);
          __syncwarp();
          if (lane < P) {
            if constexpr (DH == 1) tma_load_4d(kbuf(st) + lane * PS * 128, &tmk, &b.k_full[st], 0, 0, h, pg, kv_policy);
            else
#pragma unroll
              for (int dh = 0; dh < DH; ++dh)
                tma_load_5d(kbuf(st, dh) + lane * PS * 128, &tmk, &b.k_full[st], 0, dh, 0, h, pg, kv_policy);
          }
          if constexpr (Fmt<FMT>::SCALED) {
            copy_scales(tile, pg, st, false);
            cp_async_arrive_noinc(&b.k_full[st]);
          }
          k_issued = it + 1;
          if (lane == 0) go = mbar_wait(&b.v_empty[st], par, abort_flag, wait_ns);
          if (!__shfl_sync(0xffffffffu, go, 0)) return false;
          if (lane == 0) mbar_arrive_expect_tx(&b.v_full[st], DH * C::K_TX);
          __syncwarp();
          if (lane < P) {
            if constexpr (DH == 1) tma_load_4d(vbuf(st) + lane * PS * 128, &tmv, &b.v_full[st], 0, 0, h, pg, kv_policy);
            else
#pragma unroll
              for (int dh = 0; dh < DH; ++dh)
                tma_load_5d(vbuf(st, dh) + lane * PS * 128, &tmv, &b.v_full[st], 0, dh, 0, h, pg, kv_policy);
          }
          if constexpr (Fmt<FMT>::SCALED) {
            copy_scales(tile, pg, st, true);
            cp_async_arrive_noinc(&b.v_full[st]);
          }
          v_issued = ++it;
          return true;
        };
        int next = page_load(tb);
        for (int tile = tb; ok && tile < te; ++tile) {
          const int pg = page_check(next);
          next = page_load(tile + 1);  // rewrites the register only after the check read it
          ok = issue_tile(tile, pg);
        }
      }
      if (lane == 0) {
        if (!ok && !*abort_flag) give_up();
        if (*abort_flag) {  // every issued copy must land before the CTA may exit
          for (int k = k_issued > S ? k_issued - S : 0; k < k_issued; ++k)
            mbar_wait(&b.k_full[k % S], (k / S) & 1, &never_abort, MJ_TC_WAIT_NS);
          for (int k = v_issued > S ? v_issued - S : 0; k < v_issued; ++k)
            mbar_wait(&b.v_full[k % S], (k / S) & 1, &never_abort, MJ_TC_WAIT_NS);
        }
      }
      __syncwarp();
    } else if (warp == kWarpMma) {
      // ----------------------------------------------------- S = K . Q^T issuer
      if (lane == 0) {
        const uint32_t idesc_s = idesc_f8f6f4(Fmt<FMT>::MMA_FMT, 0u, 0u, 0u, (uint32_t)NS);
        // the abort-path probe: a bounded wait on a phase nothing completes
        bool ok = !a.abort_probe_ns || mbar_wait_rt(b.k_ready + S, 0, abort_flag, a.abort_probe_ns);
        int it = 0, jc = 0;
        for (int p = blockIdx.x; ok && p < total_jobs; p += gridDim.x) {
          int seq, tb, te, split, h, g;
          if (!job(p, seq, tb, te, split, h, g)) continue;
          ok = mbar_wait(&b.q_full[jc & 1], (jc >> 1) & 1, abort_flag, wait_ns);
          const uint32_t qaddr = smem_addr(qbuf(jc & 1));
          ++jc;
          for (int tile = tb; ok && tile < te; ++tile, ++it) {
            const int st = it % S;
            // K landed (nvfp4: converted to e4m3) and the softmax done with S buffer it & 1
            ok = mbar_wait(Fmt<FMT>::SCALED ? &b.k_ready[st] : &b.k_full[st], (it / S) & 1, abort_flag, wait_ns) &&
                 mbar_wait(&b.s_free[it & 1], ((it >> 1) & 1) ^ 1, abort_flag, wait_ns);
            if (!ok) break;
            tc_fence_after();
            const uint32_t d = tmem + (uint32_t)((it & 1) * NS);
  #pragma unroll
            for (int dh = 0; dh < DH; ++dh) {
              const uint32_t kaddr = smem_addr(kbuf(st, dh)), qa = qaddr + (uint32_t)(dh * C::QBYTES);
  #pragma unroll
              for (int k = 0; k < 4; ++k)
                mma_f8f6f4(d, smem_desc_sw128(kaddr + 32 * k, 16, ATOM), smem_desc_sw128(qa + 32 * k, 16, 1024), idesc_s,
                           dh > 0 || k > 0);
            }
            mma_commit(&b.s_full[it & 1]);
            if (!FUSED) mma_commit(&b.k_empty[st]);  // K is consumed once S is computed
          }
        }
        if (!ok && !*abort_flag) give_up();
        mma_commit(b.drain);  // all issued MMAs complete before TMEM is released
        mbar_wait(b.drain, 0, &never_abort, MJ_TC_WAIT_NS);
      }
      __syncwarp();
    } else if (warp == kWarpPv) {
      // ---------------------------------------------- O^T += V^T . P^T issuer
      if (lane == 0) {
        const uint32_t idesc_o = idesc_f8f6f4(0u, 0u, 1u, 1u, (uint32_t)NO);  // V and P both MN-major
        bool ok = true;
        int it = 0, jo = 0;
        for (int p = blockIdx.x; ok && p < total_jobs; p += gridDim.x) {
          int seq, tb, te, split, h, g;
          if (!job(p, seq, tb, te, split, h, g)) continue;
          // the job's first tile starts the accumulator fresh, once the
          // previous job's O has been read out
          ok = mbar_wait(b.o_free, (jo & 1) ^ 1, abort_flag, wait_ns);
          ++jo;
          for (int tile = tb; ok && tile < te; ++tile, ++it) {
            const int st = it % S;
            ok = mbar_wait(&b.p_full[it & 1], (it >> 1) & 1, abort_flag, wait_ns) &&
                 mbar_wait(&b.v_ready[it & 1], (it >> 1) & 1, abort_flag, wait_ns);
            if (!ok) break;
            tc_fence_after();
            const uint32_t paddr = smem_addr(pbuf(it & 1));
            // P^T is [128 s][16 B] per group of 16 rows: 8-row core matrices 128 B
            // apart along s (LBO), groups 2048 B apart (SBO); k-step = 32 s-rows.
            // Head-dim half dh accumulates into its own O block.
  #pragma unroll
            for (int dh = 0; dh < DH; ++dh) {
              const uint32_t vaddr = smem_addr(vbuf(st, dh));
              const uint32_t d = tmem + (uint32_t)(2 * NS + dh * NO);
  #pragma unroll
              for (int k = 0; k < 4; ++k)
                mma_f8f6f4(d, smem_desc_sw128(vaddr + 4 * ATOM * k, kTileBytes, ATOM),
                           smem_desc_noswz(paddr + 512 * k, 128, 2048), idesc_o, k > 0 || tile > tb);
            }
            mma_commit(&b.o_full[it & 1]);
            mma_commit(&b.v_empty[st]);
            mma_commit(&b.v_free[it & 1]);
          }
        }
        if (!ok && !*abort_flag) give_up();
        mma_commit(b.drain);
        mbar_wait(b.drain, 0, &never_abort, MJ_TC_WAIT_NS);
      }
      __syncwarp();
    } else {
      if (!(MJ_CVT_BALANCED && CVTW)) convert_role(lane);  // warp 2: converter threads 0..31
    }
  } else if (warp < C::SM0) {
    // the converter warpgroup: converter threads 32 .. CVT_ROLE - 1
    if constexpr (C::REG_LO > 0) setmaxnreg_dec<C::REG_LO>();
    convert_role(C::CVT_BASE + (int)threadIdx.x - 128);
  } else {
    if constexpr (C::REG_HI > 0) setmaxnreg_inc<C::REG_HI>();
    // -------------------------------------------------- softmax warpgroups
    const int sw = (warp - C::SM0) >> 2;              // this warpgroup: rows sw * NQP .. of the job's RT
    const int t = (threadIdx.x - C::SM0 * 32) & 127;    // TMEM lane = KV row of a tile = head-dim index
    const int wq = warp & 3;                          // TMEM lane quarter (warp % 4)
    const uint32_t lane_base = (uint32_t)(wq * 32) << 16;
    const uint32_t bar_id = 1 + sw;                   // this warpgroup's named barrier
    float* red = red_all + sw * 8 * NQP;              // [2][4][NQP]
    float* lred = lred_all + sw * 4 * NQP;            // [4][NQP]
    const int col0 = sw * NQP;                        // this warpgroup's rows within each row block
    const int h_r = a.h_q / a.h_k, q_len = a.q_len, n_q = q_len * h_r;  // rows of the whole group
    // Q rows past 3*RT (padding to the MMA's N) stay zero for the whole kernel
    if (sw == 0)
      for (int i = 0; i < 2; ++i)
        for (int dh = 0; dh < DH; ++dh)
          for (int row = 3 * RT; row < NS; ++row) qbuf(i, dh)[sw128_offset(row, t)] = 0;
    int it = 0, jc = 0;
    bool aborted = false;
    for (int p = blockIdx.x; !aborted && p < total_jobs; p += gridDim.x) {
      int seq, tb, te, split, h, g;
      if (!job(p, seq, tb, te, split, h, g)) continue;
      // ---- Q of this job: head-dim element t of each of this warpgroup's
      // query rows (group rows g*RT + sw*NQP + r), split in 3 e4m3 terms.
      // Every global read of the job start is issued before any is used (one
      // memory round trip, not one per row): padding rows read row n_q - 1
      // and are zeroed after.
      const int L = a.seq_lens[seq];
      const int nsp = a.n_splits[seq];
      const int row0 = g * RT + col0;
      float qv[DH][NQP], qm[DH][NQP];
      const int64_t qbase = (int64_t)seq * q_len * a.q_stride_tok + (int64_t)h * h_r * a.q_stride_head + t;
      auto qoff = [&](int r) {  // element offset of row r's head-dim element t
        const int R = min(row0 + r, n_q - 1);
        return qbase + (int64_t)(R / h_r) * a.q_stride_tok + (int64_t)(R % h_r) * a.q_stride_head;
      };
      auto moff = [&](int r) { return (int64_t)(h * h_r + min(row0 + r, n_q - 1) % h_r) * D + t; };
#pragma unroll
      for (int dh = 0; dh < DH; ++dh) {  // head-dim elements dh * 128 + t
        if (a.q_dtype == MJ_DT_BF16) {
          const __nv_bfloat16* q16 = reinterpret_cast<const __nv_bfloat16*>(a.q) + dh * 128;
#pragma unroll
          for (int r = 0; r < NQP; ++r) qv[dh][r] = __bfloat162float(q16[qoff(r)]);
        } else if (a.q_dtype == MJ_DT_FP16) {
          const __half* q16 = reinterpret_cast<const __half*>(a.q) + dh * 128;
#pragma unroll
          for (int r = 0; r < NQP; ++r) qv[dh][r] = __half2float(q16[qoff(r)]);
        } else {
          const float* q32 = reinterpret_cast<const float*>(a.q) + dh * 128;
#pragma unroll
          for (int r = 0; r < NQP; ++r) qv[dh][r] = q32[qoff(r)];
        }
        if (a.q_mul) {
#pragma unroll
          for (int r = 0; r < NQP; ++r) qm[dh][r] = a.q_mul[moff(r) + dh * 128];
        } else {
#pragma unroll
          for (int r = 0; r < NQP; ++r) qm[dh][r] = 1.f;
        }
      }
      float qmax = 0.f;
#pragma unroll
      for (int dh = 0; dh < DH; ++dh)
#pragma unroll
        for (int r = 0; r < NQP; ++r) {
          qv[dh][r] = row0 + r < n_q ? qv[dh][r] * qm[dh][r] : 0.f;
          qmax = fmaxf(qmax, fabsf(qv[dh][r]));
        }
      qmax = warp_max_f32(qmax);
      if (lane == 0) red[wq] = qmax;
      if (named_bar_or(bar_id, 128, *abort_flag != 0)) break;
      qmax = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
      const float qs = qmax > 0.f ? 224.f / qmax : 1.f;  // |q * qs| <= 224
#pragma unroll
      for (int dh = 0; dh < DH; ++dh) {
        unsigned char* qb = qbuf(jc & 1, dh);
#pragma unroll
        for (int r = 0; r < NQP; r += 2) {
          uint16_t hb, mb, lb;
          split3(qv[dh][r] * qs, qv[dh][r + 1] * qs, hb, mb, lb);
          store_split<RT>(qb, col0 + r, t, hb, mb, lb);
        }
      }
      fence_proxy_async_smem();
      const float kd = descale_at(a.k_descale, a.k_descale_mode, seq, h, h_k);
      const float vd = descale_at(a.v_descale, a.v_descale_mode, seq, h, h_k);
      const float c2 = a.softmax_scale * kd * kLog2e / qs;  // S (in q*qs units) -> log2 units
      if (named_bar_or(bar_id, 128, *abort_flag != 0)) break;  // Q written and fenced, red[] read
      if (t == 0) mbar_arrive(&b.q_full[jc & 1]);
      ++jc;

      // Query rows in pairs (packed f32x2 math). nm: minus the running max m'
      // in log2 units (raised lazily, see kRescaleLog2), floored so that a row
      // that has seen no key (m' = -inf) keeps nm = 3e38 and exponents of
      // -inf (p = 0, not NaN); l: this thread's partial row sums.
      // O accumulates in TMEM over the job's tiles (the PV MMA adds each tile);
      // when a row's max is raised, its O columns are rescaled in place.
      constexpr int NP = NQP / 2;
      float2 nm2[NP], l2[NP];
#pragma unroll
      for (int q = 0; q < NP; ++q) {
        nm2[q] = make_float2(3.0e38f, 3.0e38f);
        l2[q] = make_float2(0.f, 0.f);
      }
      const float2 c2v = make_float2(c2, c2);
      auto lim_of = [&](int r) {  // last key query row r may see (-1: padding row)
        const int R = row0 + r;
        return R < n_q ? (a.causal ? L - q_len + R / h_r : L - 1) : -1;
      };
      // the group's first row sees the fewest keys: a tile ending at or before
      // its limit needs no causal mask
      const int lim_min = lim_of(0);
      const uint32_t o_taddr = tmem + (uint32_t)(2 * NS) + lane_base;

      // Barrier phases. o_full[t & 1] completes once per tile t (PV_t). Before
      // writing P_t into buffer t & 1 this role waits for PV_{t-2} on it, so
      // every wait on o_full sees at most one phase pending: PV_{t-4} (and,
      // for o_full[(t-1) & 1], PV_{t-3}) completed before P_{t-2} (P_{t-1}) was
      // written, and PV_t (PV_{t+1}) needs P_t (P_{t+1}), not yet written.
      const int n = te - tb;
      for (int i = 0; i < n; ++i, ++it) {
        if (!mbar_wait(&b.s_full[it & 1], (it >> 1) & 1, abort_flag, wait_ns) && !*abort_flag) give_up();
        tc_fence_after();
        float2 x2[NP];
        const uint32_t s_taddr = tmem + (uint32_t)((it & 1) * NS) + lane_base;
        if constexpr (NQP <= 8) {
          static_assert(NWG == 1, "small row counts run one warpgroup");
          float sv[NS];
          tmem_ld_cols<NS>(s_taddr, sv);
          tmem_wait_ld();
#pragma unroll
          for (int q = 0; q < NP; ++q) x2[q] = fmul2(combine3x2<NQP>(sv, 2 * q), c2v);
        } else {  // this warpgroup's columns r, RT + r, 2 RT + r of 16 query rows: one wait
          static_assert(NQP == 16, "wide variants run 16 rows per warpgroup");
          float hv[16], mv[16], lv[16];
          tmem_ld16(s_taddr + col0, hv);
          tmem_ld16(s_taddr + RT + col0, mv);
          tmem_ld16(s_taddr + 2 * RT + col0, lv);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 16; k += 2) {
            const float2 hi = make_float2(hv[k], hv[k + 1]), mid = make_float2(mv[k], mv[k + 1]),
                         lo = make_float2(lv[k], lv[k + 1]);
            x2[k / 2] = fmul2(
                ffma2(lo, make_float2(0.00390625f, 0.00390625f), ffma2(mid, make_float2(0.0625f, 0.0625f), hi)), c2v);
          }
        }
        tc_fence_before();
        mbar_arrive(&b.s_free[it & 1]);
        const int j0 = (tb + i) * kTileRows, j = j0 + t;  // this thread's KV row
        const bool edge = j0 + kTileRows - 1 > lim_min;  // some row sees only part of this tile
        if (edge) {  // rare (the tiles at a causal tail): recompute the limits
#pragma unroll
          for (int q = 0; q < NP; ++q) {
            if (j > lim_of(2 * q)) x2[q].x = -INFINITY;
            if (j > lim_of(2 * q + 1)) x2[q].y = -INFINITY;
          }
        }
        // From here x2 holds the exponents d = s - m'. The job's first tile
        // always sets the running max; later ones test the largest exponent.
        bool grow = i == 0;
        if (!grow) {
          float dmax = -INFINITY;
#pragma unroll
          for (int q = 0; q < NP; ++q) {
            x2[q] = fadd2(x2[q], nm2[q]);
            dmax = fmaxf(dmax, fmaxf(x2[q].x, x2[q].y));
          }
          grow = dmax > kRescaleLog2 + kLog2PScale;
        }
        // one barrier per tile: a uniform vote on "some score outgrew its row's
        // max" (or abort); only then do the rows exchange their tile maxima
        if (named_bar_or(bar_id, 128, grow || *abort_flag != 0)) {
          if (named_bar_or(bar_id, 128, *abort_flag != 0)) {
            aborted = true;
            break;
          }
          if (i > 0) {  // back to scores: m' is finite here for every row that sees a key
#pragma unroll
            for (int q = 0; q < NP; ++q) x2[q] = fadd2(x2[q], make_float2(-nm2[q].x, -nm2[q].y));
          }
          float* rd = red + (it & 1) * 4 * NQP;
#pragma unroll
          for (int q = 0; q < NP; ++q) {
            const float w0 = warp_max_f32(x2[q].x), w1 = warp_max_f32(x2[q].y);
            if (lane == 0) {
              rd[wq * NQP + 2 * q] = w0;
              rd[wq * NQP + 2 * q + 1] = w1;
            }
          }
          named_bar_sync(bar_id, 128);
          // lane r < NQP takes row r's maximum over the four warps and hands it
          // round (rather than every lane loading all 4 x NQP, which the
          // compiler hoists into as many live registers)
          const float mine = lane < NQP ? fmaxf(fmaxf(rd[lane], rd[NQP + lane]), fmaxf(rd[2 * NQP + lane], rd[3 * NQP + lane])) : 0.f;
          float cc[NQP];  // correction of each row's earlier sums: 2^(m_old - m_new)
#pragma unroll
          for (int r = 0; r < NQP; ++r) {
            const float mt = __shfl_sync(0xffffffffu, mine, r) - kLog2PScale;
            float& nmr = (r & 1) ? nm2[r >> 1].y : nm2[r >> 1].x;
            float& lr = (r & 1) ? l2[r >> 1].y : l2[r >> 1].x;
            cc[r] = 1.f;
            if (mt > -nmr) {  // from a row with no key yet (nm = 3e38): 2^-inf = 0
              cc[r] = exp2_approx(-nmr - mt);
              lr *= cc[r];
              nmr = -mt;
            }
          }
          if (i >= 1) {  // O holds tiles tb .. tb+i-1: once PV_{it-1} lands, scale its rows
            if (!mbar_wait(&b.o_full[(it - 1) & 1], ((it - 1) >> 1) & 1, abort_flag, wait_ns) && !*abort_flag)
              give_up();
            tc_fence_after();
            if constexpr (NWG == 1) {  // the three row blocks are contiguous: 3 * NQP columns
#pragma unroll
              for (int dh = 0; dh < DH; ++dh)
#pragma unroll
                for (int c = 0; c < 3 * NQP; c += 8) {
                  float ov[8];
                  tmem_ld8(o_taddr + dh * NO + c, ov);
                  tmem_wait_ld();
#pragma unroll
                  for (int k = 0; k < 8; ++k)
                    if (c + k < 3 * NQP) ov[k] *= cc[(c + k) % NQP];
                  tmem_st8(o_taddr + dh * NO + c, ov);
                }
            } else {  // this warpgroup's NQP columns of each row block
#pragma unroll
              for (int blk = 0; blk < 3; ++blk)
#pragma unroll
                for (int c = 0; c < NQP; c += 8) {
                  float ov[8];
                  tmem_ld8(o_taddr + blk * RT + col0 + c, ov);
                  tmem_wait_ld();
#pragma unroll
                  for (int k = 0; k < 8; ++k) ov[k] *= cc[c + k];
                  tmem_st8(o_taddr + blk * RT + col0 + c, ov);
                }
            }
            tmem_wait_st();
          }
#pragma unroll
          for (int q = 0; q < NP; ++q) x2[q] = fadd2(x2[q], nm2[q]);  // exponents under the new max
        }
        // P: three e4m3 terms per row, this thread's KV row s = t packed as the
        // 16-byte row s of each MN-major group (N rows hi | mid | lo | padding)
        // words of this thread's P bytes: term k of row r at byte k * NQP + r
        constexpr int NW = NWG == 1 ? NO / 4 : 3 * NQP / 4;
        uint32_t w[NW];
#pragma unroll
        for (int k = 0; k < NW; ++k) w[k] = 0u;
#pragma unroll
        for (int q = 0; q < NP; ++q) {
          const float2 pv = make_float2(exp2_approx(x2[q].x), exp2_approx(x2[q].y));
          l2[q] = fadd2(l2[q], pv);
          uint16_t hb, mb, lb;
          split3x2(pv, hb, mb, lb);
          const int r = 2 * q, sh = 16 * (q & 1);
          w[r >> 2] |= (uint32_t)hb << sh;
          w[(NQP + r) >> 2] |= (uint32_t)mb << sh;
          w[(2 * NQP + r) >> 2] |= (uint32_t)lb << sh;
        }
        // buffer it & 1 was read by PV_{it-2}: it must have completed
        if (it >= 2 && !mbar_wait(&b.o_full[it & 1], ((it >> 1) & 1) ^ 1, abort_flag, wait_ns) && !*abort_flag)
          give_up();
        unsigned char* pb = pbuf(it & 1);
        if constexpr (NWG == 1) {  // the whole operand row: groups 0 .. NO/16
#pragma unroll
          for (int g = 0; g < NO / 16; ++g)
            *reinterpret_cast<uint4*>(pb + g * 2048 + t * 16) = make_uint4(w[4 * g], w[4 * g + 1], w[4 * g + 2], w[4 * g + 3]);
        } else {  // this warpgroup's 16-row groups of each term block
#pragma unroll
          for (int k = 0; k < 3; ++k)
#pragma unroll
            for (int j = 0; j < NQP / 16; ++j) {
              const int g = (k * RT + col0) / 16 + j, wi = (k * NQP + 16 * j) / 4;
              *reinterpret_cast<uint4*>(pb + g * 2048 + t * 16) = make_uint4(w[wi], w[wi + 1], w[wi + 2], w[wi + 3]);
            }
        }
        fence_proxy_async_smem();
        tc_fence_before();  // orders a rescale's TMEM stores before PV_it
        mbar_arrive(&b.p_full[it & 1]);
        if constexpr (C::SM_CONVERTS) {  // this warpgroup's share of the V conversion
          const int st = it % S;
          if (!FUSED && !mbar_wait(&b.v_full[st], (it / S) & 1, abort_flag, wait_ns) && !*abort_flag) give_up();
          unsigned char* vb = vbuf(st);
#pragma unroll 2
          for (int c = C::CVT_ROLE + sw * 128 + t; c < kTileBytes / 16; c += C::CVT_THREADS) {
            uint4* q = reinterpret_cast<uint4*>(vb + vchunk(c));
            *q = Fmt<FMT>::convert(*q);
          }
          fence_proxy_async_smem();
          mbar_arrive(&b.v_ready[it & 1]);
        } else if constexpr (C::SM_CVT_VHI) {  // head_dim 256: the second half of this tile's V
          const int st = it % S;
          if (!FUSED && !mbar_wait(&b.v_full[st], (it / S) & 1, abort_flag, wait_ns) && !*abort_flag) give_up();
#pragma unroll 2
          for (int g = DH * (kTileBytes / 16) - C::SM_CHUNKS + t; g < DH * (kTileBytes / 16); g += 128) {
            uint4* q = reinterpret_cast<uint4*>(vbuf(st, g >> 10) + vchunk(g & 1023));
            *q = Fmt<FMT>::convert(*q);
          }
          fence_proxy_async_smem();
          mbar_arrive(&b.v_ready[it & 1]);
        } else if constexpr (C::SM_CVT_V) {  // nvfp4: this tile's V, rows past the sequence zeroed
          const int st = it % S;
          if (!FUSED && !mbar_wait(&b.v_full[st], (it / S) & 1, abort_flag, wait_ns) && !*abort_flag) give_up();
          nvfp4_tile(vbuf(st), vscl(st), L - j0, t, 128);
          fence_proxy_async_smem();
          mbar_arrive(&b.v_ready[it & 1]);
        }
      }
      if (aborted) break;

      // ---- epilogue: l per query row (sum of the per-thread partials), O from TMEM
#pragma unroll
      for (int r = 0; r < NQP; ++r) {
        float x = (r & 1) ? l2[r >> 1].y : l2[r >> 1].x;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
        if (lane == 0) lred[wq * NQP + r] = x;
      }
      if (!mbar_wait(&b.o_full[(it - 1) & 1], ((it - 1) >> 1) & 1, abort_flag, wait_ns) && !*abort_flag)
        give_up();
      tc_fence_after();
      float orow[DH][NQP];  // this thread's head-dim elements of every row: hi + mid / 16 + lo / 256
#pragma unroll
      for (int dh = 0; dh < DH; ++dh)
#pragma unroll
        for (int c = 0; c < NQP; c += 8) {
          float hv[8], mv[8], lv[8];
          tmem_ld8(o_taddr + dh * NO + col0 + c, hv);
          tmem_ld8(o_taddr + dh * NO + RT + col0 + c, mv);
          tmem_ld8(o_taddr + dh * NO + 2 * RT + col0 + c, lv);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 8 && c + k < NQP; ++k) orow[dh][c + k] = hv[k] + mv[k] * 0.0625f + lv[k] * 0.00390625f;
        }
      tc_fence_before();
      mbar_arrive(b.o_free);  // the next job's first PV may overwrite O
      if (named_bar_or(bar_id, 128, *abort_flag != 0)) {
        aborted = true;
        break;
      }
      const bool final_out = nsp <= 1;
      const float vscale = Fmt<FMT>::V_UNSCALE * vd;
      const int qi0 = row0 / h_r, rr0 = row0 % h_r;
      auto qh_of = [&](int r) { return h * h_r + (rr0 + r) % h_r; };
      auto tok_of = [&](int r) { return (int64_t)seq * q_len + qi0 + (rr0 + r) / h_r; };
      if (!final_out && (split >= a.max_splits || seq >= a.part_seqs || !a.o_part)) {
        if (t == 0) flag(a.status, MJ_DEV_BAD_SPLIT);
      } else {
        // O rows: normalized, times the V channel scales (final) -- the o_mul
        // reads are issued together, the dtype branch taken once per job
#pragma unroll
        for (int dh = 0; dh < DH; ++dh) {  // head-dim element e = dh * 128 + t
          const int e = dh * 128 + t;
          float o[NQP];
#pragma unroll
          for (int r = 0; r < NQP; ++r) {
            const float lt = lred[r] + lred[NQP + r] + lred[2 * NQP + r] + lred[3 * NQP + r];
            o[r] = lt > 0.f ? orow[dh][r] * __fdividef(vscale, lt) : 0.f;
          }
          if (final_out && a.o_mul) {
            float om[NQP];
#pragma unroll
            for (int r = 0; r < NQP; ++r) om[r] = a.o_mul[(int64_t)qh_of(min(r, n_q - 1 - row0)) * D + e];
#pragma unroll
            for (int r = 0; r < NQP; ++r) o[r] *= om[r];
          }
          if (final_out) {
            if (a.o_dtype == MJ_DT_BF16) {
              __nv_bfloat16* o16 = reinterpret_cast<__nv_bfloat16*>(a.o);
#pragma unroll
              for (int r = 0; r < NQP; ++r)
                if (row0 + r < n_q) o16[tok_of(r) * a.o_stride_tok + qh_of(r) * a.o_stride_head + e] = __float2bfloat16_rn(o[r]);
            } else {
#pragma unroll
              for (int r = 0; r < NQP; ++r)
                if (row0 + r < n_q) store_elem(a.o, tok_of(r) * a.o_stride_tok + qh_of(r) * a.o_stride_head + e, a.o_dtype, o[r]);
            }
          } else {
            const int64_t prow = (((int64_t)split * a.part_seqs + seq) * h_k + h) * n_q + row0;
#pragma unroll
            for (int r = 0; r < NQP; ++r)
              if (row0 + r < n_q) a.o_part[(prow + r) * D + e] = o[r];
          }
        }
        if (t < NQP && row0 + t < n_q) {  // LSE (natural log) of row t: thread t writes it
          float lt = 0.f, mr = 0.f;
#pragma unroll
          for (int r = 0; r < NQP; ++r)
            if (r == t) {
              lt = lred[r] + lred[NQP + r] + lred[2 * NQP + r] + lred[3 * NQP + r];
              mr = -((r & 1) ? nm2[r >> 1].y : nm2[r >> 1].x);
            }
          const float lse = lt > 0.f ? (mr + log2f(lt)) * kLn2 : -INFINITY;
          if (!final_out) a.lse_part[(((int64_t)split * a.part_seqs + seq) * h_k + h) * n_q + row0 + t] = lse;
          else if (a.lse) a.lse[tok_of(t) * a.h_q + qh_of(t)] = lse;
        }
      }
      // In-kernel split merge (one warpgroup per CTA, whose threads all take
      // the same path): every job of a split (sequence, KV head, row group)
      // counts itself in; the last one merges the partials and writes the
      // final O / LSE, and puts the counter back to zero for the next launch.
      if constexpr (NWG == 1) {
        if (!final_out && a.merge_counters && a.max_splits <= kMergeMaxSplits) {
          __threadfence();  // this job's partials, visible device-wide before it counts
          named_bar_sync(bar_id, 128);
          int* last_flag = reinterpret_cast<int*>(sm + C::MISC_OFF + 12);
          if (t == 0) {
            int* ctr = a.merge_counters + ((int64_t)seq * h_k + h) * n_rg + g;
            const int last = atomicAdd(ctr, 1) == nsp - 1;
            if (last) atomicExch(ctr, 0);
            *last_flag = last;
          }
          named_bar_sync(bar_id, 128);
          if (*last_flag && seq < a.part_seqs) {
            __threadfence();
            // every partial LSE of the group's rows, one per thread, into shared
            // memory; then each thread merges its head-dim element of every row,
            // the O partial reads of a row issued together
            constexpr int MAXS = kMergeMaxSplits;
            const int ns = min(nsp, a.max_splits);
            const int64_t stride = (int64_t)a.part_seqs * h_k * n_q;
            const int64_t base = ((int64_t)seq * h_k + h) * n_q + row0;
            // scratch: the P buffer of tile it - 2, whose PV completed (PBYTES >= MAXS * NQP * 4)
            float* lsm = reinterpret_cast<float*>(sm + C::P_OFF + (it & 1) * C::PBYTES);
            for (int i = t; i < ns * NQP; i += 128) {
              const int k = i / NQP, r = i % NQP;
              lsm[i] = row0 + r < n_q ? __ldcg(a.lse_part + k * stride + base + r) : -INFINITY;
            }
            named_bar_sync(bar_id, 128);
            for (int r = 0; r < NQP; ++r) {
              if (row0 + r >= n_q) break;
              float m = -INFINITY;
              for (int k = 0; k < ns; ++k) m = fmaxf(m, lsm[k * NQP + r]);
              float den = 0.f;
#pragma unroll
              for (int dh = 0; dh < DH; ++dh) {  // head-dim element e = dh * 128 + t
                const int e = dh * 128 + t;
                float ov[MAXS];
#pragma unroll
                for (int k = 0; k < MAXS; ++k) ov[k] = k < ns ? __ldcg(a.o_part + (k * stride + base + r) * D + e) : 0.f;
                float acc = 0.f;
                den = 0.f;
                if (m != -INFINITY) {
#pragma unroll
                  for (int k = 0; k < MAXS; ++k)
                    if (k < ns) {
                      const float w = __expf(lsm[k * NQP + r] - m);
                      den += w;
                      acc = fmaf(w, ov[k], acc);
                    }
                }
                float o = den > 0.f ? acc / den : 0.f;
                if (a.o_mul) o *= a.o_mul[(int64_t)qh_of(r) * D + e];
                store_elem(a.o, tok_of(r) * a.o_stride_tok + qh_of(r) * a.o_stride_head + e, a.o_dtype, o);
              }
              if (t == 0 && a.lse) a.lse[tok_of(r) * a.h_q + qh_of(r)] = den > 0.f ? m + __logf(den) : -INFINITY;
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
// launch templates (instantiated once per KV format, inst_<format>.cu)
// ---------------------------------------------------------------------------
namespace mj {

// One process may drive several GPUs: the shared-memory attributes are set,
// and the resident-CTA count is derived, once per (kernel variant, device).
constexpr int kMaxDevices = 64;
std::mutex& tc_init_mutex();

// Launch (or, when `dry`, only prepare and check) one tensor-core variant.
// cudaErrorNotSupported: this variant's register split does not fit the
// launch allocation on this build; the caller tries the next variant.
template <int FMT, int NQP, int NWG, int CVTW, bool FUSED, int DH = 1>
static cudaError_t launch_tc_t(const mj_decode_args& a, const CUtensorMap& mk, const CUtensorMap& mv,
                               cudaStream_t stream, bool dry) {
  using C = tc::Cfg<FMT, NQP, NWG, CVTW, DH>;
  auto kern = tc::decode_tc_kernel<FMT, NQP, NWG, CVTW, FUSED, DH>;
  const int smem = C::SMEM;
  static std::atomic<int> slots_of[kMaxDevices];  // resident CTAs per device; 0 unknown, -1 unusable
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int slots = slots_of[dev].load(std::memory_order_acquire);
  if (!slots) {
    std::lock_guard<std::mutex> lock(tc_init_mutex());
    slots = slots_of[dev].load(std::memory_order_acquire);
    if (!slots) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
      // without a carveout preference the occupancy is computed for a smaller
      // shared-memory partition and one CTA per SM would be assumed
      e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
      if (e != cudaSuccess) return e;
      // resident CTAs per SM from the device limits: shared memory (with the
      // per-block reserve), registers, and the 512 TMEM columns of an SM
      int sms = 0, smem_sm = 0, reserve = 0, regs_sm = 0;
      cudaFuncAttributes fa;
      if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
      if ((e = cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev)) != cudaSuccess) return e;
      if ((e = cudaDeviceGetAttribute(&reserve, cudaDevAttrReservedSharedMemoryPerBlock, dev)) != cudaSuccess) return e;
      if ((e = cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev)) != cudaSuccess) return e;
      if ((e = cudaFuncGetAttributes(&fa, kern)) != cudaSuccess) return e;
      if (C::REG_POOL > fa.numRegs * C::THREADS) {
        // a register split must fit the CTA's launch allocation, or the
        // increasing warpgroups would wait for registers that never come
        slots = -1;
      } else {
        int occ = smem_sm / (smem + (int)fa.sharedSizeBytes + reserve);
        const int regs_cta = ((fa.numRegs + 7) / 8) * 8 * C::THREADS;
        occ = occ < regs_sm / regs_cta ? occ : regs_sm / regs_cta;
        occ = occ < 512 / C::TMEM_COLS ? occ : 512 / C::TMEM_COLS;
        occ = occ < C::CTAS_PER_SM ? occ : C::CTAS_PER_SM;  // __launch_bounds__ min blocks
        slots = sms * (occ > 0 ? occ : 1);
      }
      slots_of[dev].store(slots, std::memory_order_release);
    }
  }
  if (slots < 0) return cudaErrorNotSupported;
  if (dry) return cudaSuccess;
  const int n_q = a.q_len * (a.h_q / a.h_k);
  const int64_t jobs = (int64_t)a.num_work * a.h_k * ((n_q + C::RT - 1) / C::RT);
  const unsigned grid = (unsigned)(jobs < slots ? jobs : slots);
  return launch_kernel(kern, dim3(grid), dim3(C::THREADS), (size_t)smem, stream, a, mk, mv);
}

// Variant by query rows per KV head (n_q): one warpgroup of 4, 8 or 16 rows
// (two CTAs per SM; narrow formats add a converter warpgroup), or two / three
// warpgroups of 16 rows in one CTA per SM that read each KV tile once for up
// to 48 rows (row groups of 48 beyond). A variant whose register split the
// launch cannot cover is skipped for the next one down.
template <int FMT, int NQP, bool FUSED>
static cudaError_t launch_one_wg(const mj_decode_args& a, const CUtensorMap& mk, const CUtensorMap& mv,
                                 cudaStream_t stream, bool dry) {
  if constexpr (tc::Fmt<FMT>::NARROW) {
    cudaError_t e = launch_tc_t<FMT, NQP, 1, 1, FUSED>(a, mk, mv, stream, dry);
    if (e != cudaErrorNotSupported) return e;
  }
  return launch_tc_t<FMT, NQP, 1, 0, FUSED>(a, mk, mv, stream, dry);
}

template <int FMT, bool FUSED>
static cudaError_t dispatch_fmt(const mj_decode_args& a, int n_q, const CUtensorMap& mk, const CUtensorMap& mv,
                                cudaStream_t stream, bool dry) {
  if constexpr (tc::Fmt<FMT>::SCALED) {  // nvfp4: the variants with a converter warpgroup only
    if (n_q <= 4) return launch_tc_t<FMT, 4, 1, 1, FUSED>(a, mk, mv, stream, dry);
    if (n_q <= 8) return launch_tc_t<FMT, 8, 1, 1, FUSED>(a, mk, mv, stream, dry);
    if (n_q <= 16) return launch_tc_t<FMT, 16, 1, 1, FUSED>(a, mk, mv, stream, dry);
    return launch_tc_t<FMT, 16, 3, 1, FUSED>(a, mk, mv, stream, dry);
  } else {
    if (n_q <= 4) return launch_one_wg<FMT, 4, FUSED>(a, mk, mv, stream, dry);
    if (n_q <= 8) return launch_one_wg<FMT, 8, FUSED>(a, mk, mv, stream, dry);
    if (n_q <= 16) return launch_one_wg<FMT, 16, FUSED>(a, mk, mv, stream, dry);
    if (n_q <= 32) return launch_tc_t<FMT, 16, 2, 0, FUSED>(a, mk, mv, stream, dry);
    cudaError_t e = cudaErrorNotSupported;
    if constexpr (tc::Fmt<FMT>::NARROW) e = launch_tc_t<FMT, 16, 3, 1, FUSED>(a, mk, mv, stream, dry);
    if (e == cudaErrorNotSupported) e = launch_tc_t<FMT, 16, 3, 0, FUSED>(a, mk, mv, stream, dry);
    if (e == cudaErrorNotSupported) return launch_tc_t<FMT, 16, 2, 0, FUSED>(a, mk, mv, stream, dry);
    return e;
  }
}

// head_dim 256: one warpgroup of 4, 8 or 16 rows (row groups of 16 beyond),
// one CTA per SM; narrow formats (nvfp4 included) with a converter
// warpgroup, fp8 without.
template <int FMT, bool FUSED>
static cudaError_t dispatch_fmt_d256(const mj_decode_args& a, int n_q, const CUtensorMap& mk, const CUtensorMap& mv,
                                     cudaStream_t stream, bool dry) {
  constexpr int CV = tc::Fmt<FMT>::NARROW ? 1 : 0;
  if (n_q <= 4) return launch_tc_t<FMT, 4, 1, CV, FUSED, 2>(a, mk, mv, stream, dry);
  if (n_q <= 8) return launch_tc_t<FMT, 8, 1, CV, FUSED, 2>(a, mk, mv, stream, dry);
  return launch_tc_t<FMT, 16, 1, CV, FUSED, 2>(a, mk, mv, stream, dry);
}

// The entry the host side (decode_tc.cu) calls for one KV format.
template <int FMT>
cudaError_t launch_tc_fmt(const mj_decode_args& a, int n_q, bool fused, const CUtensorMap& mk, const CUtensorMap& mv,
                          cudaStream_t stream, bool dry) {
  if (a.head_size == 256)
    return fused ? dispatch_fmt_d256<FMT, true>(a, n_q, mk, mv, stream, dry)
                 : dispatch_fmt_d256<FMT, false>(a, n_q, mk, mv, stream, dry);
  return fused ? dispatch_fmt<FMT, true>(a, n_q, mk, mv, stream, dry)
               : dispatch_fmt<FMT, false>(a, n_q, mk, mv, stream, dry);
}

}  // namespace mj
