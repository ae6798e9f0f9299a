// B200 (sm_100a) fused sampling / speculative-verification kernels behind the C ABI of
// include/sonic_b200.h.
//
// Singular and top-k calls are one launch; a multistep call is two (the rows' streaming
// pass, then one CTA per request for merge and verification). Each row is cut into S
// column splits, one 256-thread CTA per split. A CTA streams its split from HBM exactly
// once: bulk (TMA) copies of 2048-column chunks fill a shared-memory ring that is refilled
// as soon as every warp has consumed a stage, so several chunks are always in flight. Each
// thread turns 8 columns into processed bf16 logits with packed bf16x2 arithmetic and keeps
// the ones at or above a rising cut in sorted per-warp top-128 lists (fed through per-warp
// shared-memory queues). The split's exact top-128 (or, for greedy rows, its single best
// key) goes to the workspace, sorted. The last CTA of a singular or top-k row (per-row
// ticket in the workspace) merges the S sorted lists with warp bitonic merges and runs the
// selection. No host sync anywhere.
//
// Reference kernels covered (tachyontrails/sonic-sampler, src/sonic_sampler/):
//   ops/prologue.py:272-472   bitpacked_reduction_kernel (processors + tile candidates)
//   ops/topk/bitpack.py:99    bitpacked_reduction_kernel (plain top-k)
//   ops/topk/unpack.py:312    merge_unpack_kernel
//   ops/singular.py:154       cumulative_selection_kernel
//   ops/multistep.py:76       cumulative_unpack_kernel
//   ops/verify.py:244         chain_speculative_verification_kernel

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

#include "../../include/sonic_b200.h"
#include "common.cuh"

namespace sonic {

constexpr int NT = 256;                    // threads per CTA
constexpr int VPT = 8;                     // consecutive columns per thread per chunk
constexpr int CH = NT * VPT;               // columns per chunk (single-row kernels)
constexpr int STAGES = 4;                  // bulk-copy ring depth (stages of every stream)
constexpr int TARGET_CTAS = 296;           // 148 SMs x 2 resident CTAs: one wave
constexpr int MAX_SPLIT_COLS = 65536;      // columns of a split in one-wave grids
constexpr int SPLIT_MAX_COLS = 256 * CH;   // columns one CTA of the general kernel can cover
constexpr int WIDE_GROUPS = 2;             // groups a warp takes from one wide chunk (greedy rows)
constexpr int WIDE_GROUPS_LONG = 4;        // the same for CTAs of at least WIDE_LONG_COLS columns
constexpr int WIDE_LONG_COLS = 32 * CH;
constexpr int MAX_SPLITS = 32;
constexpr uint32_t WAIT_LIMIT = 1u << 22;  // polls of a bulk-copy barrier before giving up
constexpr int MS_MAX_STEPS = SONIC_MAX_LOOKAHEAD + 1;

enum LoadMode { kTma = 0, kVec = 1, kScalar = 2 };

struct Plan {
  int splits;
  int cols;
};

// Column split of a unit (row or request) of V columns; a pure function of the shapes, so
// the workspace size never depends on the device.
static Plan split_plan(int64_t units, int64_t V, int chunk) {
  if (V <= 0) return Plan{1, chunk};  // no columns: callers reject such calls before launching
  int64_t s = units > 0 ? TARGET_CTAS / units : 1;
  s = std::max<int64_t>(s, 1);
  s = std::max<int64_t>(s, (V + MAX_SPLIT_COLS - 1) / MAX_SPLIT_COLS);
  s = std::min<int64_t>(s, MAX_SPLITS);
  int64_t cols = (V + s - 1) / s;
  cols = (cols + chunk - 1) / chunk * chunk;
  cols = std::min<int64_t>(cols, MAX_SPLIT_COLS);
  Plan p;
  p.splits = (int)((V + cols - 1) / cols);
  p.cols = (int)cols;
  return p;
}

// workspace: [256-byte header: u32 error word at offset 0] | [rows][splits][128] u64 sorted
// candidate keys | [units] u32 tickets. The error word sits at a fixed offset so that
// sonic_workspace_error() can read it without the call's shapes.
constexpr size_t kWsHeader = 256;

struct Workspace {
  uint64_t* cand;
  uint32_t* tickets;
  uint32_t* error;
};

static size_t workspace_bytes(int64_t rows, int64_t units, int64_t splits) {
  if (units <= 0) return 0;
  const size_t cand = (size_t)rows * splits * kMaxK * sizeof(uint64_t);
  const size_t tick = ((size_t)units * sizeof(uint32_t) + 255) / 256 * 256;
  return kWsHeader + cand + tick;
}

// The library's own scratch (sonic_fused_singular_static), held by every GPU that loads the
// library: its first 4 bytes are also the error word of the calls that take no workspace.
constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

static Workspace carve(void* base, int64_t rows, int64_t units, int64_t splits) {
  Workspace w;
  w.error = (uint32_t*)base;
  w.cand = (uint64_t*)((char*)base + kWsHeader);
  w.tickets = (uint32_t*)((char*)w.cand + (size_t)rows * splits * kMaxK * sizeof(uint64_t));
  return w;
}

// ---------------------------------------------------------------------------------------
// small device utilities
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ int64_t load_index(const void* p, int32_t dtype, int64_t i) {
  return dtype == SONIC_DTYPE_I64 ? ((const int64_t*)p)[i] : (int64_t)((const int32_t*)p)[i];
}

__device__ __forceinline__ uint64_t ldcg64(const uint64_t* p) {
  return (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(p));
}

__device__ __forceinline__ uint32_t ldcg32(const uint32_t* p) { return __ldcg(p); }

__device__ __forceinline__ void stcg64(uint64_t* p, uint64_t v) {
  __stcg(reinterpret_cast<unsigned long long*>(p), (unsigned long long)v);
}

__device__ __forceinline__ uint4 ld_stream(const void* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void store_float(void* base, int32_t dtype, int64_t i, float x) {
  if (dtype == SONIC_DTYPE_F32)
    ((float*)base)[i] = x;
  else
    ((uint16_t*)base)[i] = f2bf(x);
}

__device__ __forceinline__ int64_t load_slot(const SonicSamplingParams& P, int64_t unit) {
  return P.slot_mapping ? load_index(P.slot_mapping, P.slot_dtype, unit) : unit;
}

// Which aux streams a row needs (reference ops/prologue.py:378-447).
struct Needs {
  bool proc, g, dec, ctx, bias, temp;
};

// Per-row constants of the logit processors.
struct RowConsts {
  uint32_t ind;
  Needs nd;
  float rep, rrep;        // multiplicative penalty and RN(1/penalty)
  bool rep_fast;          // v / rep == v * rrep after bf16 rounding (penalty in [2^-8, 2^8])
  uint32_t freq2, pres2;  // bf16 penalties in both halves
  float temp, rtemp;
  bool temp_fast;
  bool fast;  // stochastic row whose final value is a monotone map of the post-bias value
  bool decr;  // fast row whose penalties never raise a logit (given non-negative counts)
};

// For bf16 v and a bf16 divisor t in [2^-8, 2^8], bf16(v / t) == bf16(v * RN(1/t)): the exact
// quotient of two 8-bit significands is never within 2^-16 (relative) of a bf16 rounding
// midpoint, far above the 2-ulp fp32 error of the reciprocal product (checked exhaustively
// over all bf16 v and t in that range).
__device__ __forceinline__ bool recip_exact_range(float t) { return t >= 0.00390625f && t <= 256.0f; }

__device__ __forceinline__ RowConsts row_consts(const SonicSamplingParams& P, int64_t slot, uint32_t ind) {
  RowConsts rc;
  rc.ind = ind;
  Needs& n = rc.nd;
  n.proc = (ind & 0x1F) != 0;
  n.g = n.proc && P.grammar && (ind & 0x1);
  n.dec = n.proc && P.decode_counts && (ind & 0xE);
  n.ctx = n.dec && P.context_counts && (ind & 0x2);
  n.bias = n.proc && P.bias && (ind & 0x10);
  n.temp = (ind & 0x20) != 0;
  rc.rep = (n.ctx && P.repetition) ? bf2f(P.repetition[slot]) : 1.0f;
  rc.rrep = __frcp_rn(rc.rep);
  rc.rep_fast = recip_exact_range(rc.rep);
  const uint32_t f = (P.frequency && (ind & 0x4)) ? P.frequency[slot] : 0u;
  const uint32_t p = (P.presence && (ind & 0x8)) ? P.presence[slot] : 0u;
  rc.freq2 = f | (f << 16);
  rc.pres2 = p | (p << 16);
  rc.temp = (P.temperature && n.temp) ? bf2f(P.temperature[slot]) : 1.0f;
  rc.rtemp = __frcp_rn(rc.temp);
  rc.temp_fast = recip_exact_range(rc.temp);
  // The fast path skips the penalties where both counts are zero; that is exact unless a
  // negative frequency / presence penalty turns a -0.0 logit into +0.0.
  const bool neg_pen = n.dec && (((ind & 0x4) && (f & 0x8000u)) || ((ind & 0x8) && (p & 0x8000u)));
  const bool temp_ok = !n.temp || (rc.temp > 0.0f && rc.temp <= 3.3895313892515355e+38f);
  rc.fast = !(ind & 0x40) && !neg_pen && temp_ok;
  rc.decr = rc.fast && (!n.ctx || rc.rep >= 1.0f);
  return rc;
}

// Every per-slot scalar a row may read, loaded in one batch: the loads depend on the slot
// only (a NULL buffer reads as its neutral value), so they share one memory round trip
// instead of a chain slot -> indicator -> penalties -> masking parameters.
struct SlotScalars {
  uint32_t ind;
  uint16_t rep, freq, pres, temp, top_p, min_p;
  int32_t top_k, top_logprobs;
};

__device__ __forceinline__ SlotScalars load_slot_scalars(const SonicSamplingParams& P, int64_t slot) {
  SlotScalars s;
  s.ind = P.indicators[slot];
  s.rep = P.repetition ? P.repetition[slot] : (uint16_t)0x3f80u;
  s.freq = P.frequency ? P.frequency[slot] : (uint16_t)0;
  s.pres = P.presence ? P.presence[slot] : (uint16_t)0;
  s.temp = P.temperature ? P.temperature[slot] : (uint16_t)0x3f80u;
  s.top_p = P.top_p ? P.top_p[slot] : (uint16_t)0;
  s.min_p = P.min_p ? P.min_p[slot] : (uint16_t)0;
  s.top_k = P.top_k ? P.top_k[slot] : 0;
  s.top_logprobs = P.top_logprobs ? P.top_logprobs[slot] : 0;
  return s;
}

// row_consts from preloaded scalars (same result as row_consts(P, slot, s.ind))
__device__ __forceinline__ RowConsts row_consts(const SonicSamplingParams& P, const SlotScalars& s) {
  RowConsts rc;
  const uint32_t ind = s.ind;
  rc.ind = ind;
  Needs& n = rc.nd;
  n.proc = (ind & 0x1F) != 0;
  n.g = n.proc && P.grammar && (ind & 0x1);
  n.dec = n.proc && P.decode_counts && (ind & 0xE);
  n.ctx = n.dec && P.context_counts && (ind & 0x2);
  n.bias = n.proc && P.bias && (ind & 0x10);
  n.temp = (ind & 0x20) != 0;
  rc.rep = (n.ctx && P.repetition) ? bf2f(s.rep) : 1.0f;
  rc.rrep = __frcp_rn(rc.rep);
  rc.rep_fast = recip_exact_range(rc.rep);
  const uint32_t f = (P.frequency && (ind & 0x4)) ? s.freq : 0u;
  const uint32_t p = (P.presence && (ind & 0x8)) ? s.pres : 0u;
  rc.freq2 = f | (f << 16);
  rc.pres2 = p | (p << 16);
  rc.temp = (P.temperature && n.temp) ? bf2f(s.temp) : 1.0f;
  rc.rtemp = __frcp_rn(rc.temp);
  rc.temp_fast = recip_exact_range(rc.temp);
  const bool neg_pen = n.dec && (((ind & 0x4) && (f & 0x8000u)) || ((ind & 0x8) && (p & 0x8000u)));
  const bool temp_ok = !n.temp || (rc.temp > 0.0f && rc.temp <= 3.3895313892515355e+38f);
  rc.fast = !(ind & 0x40) && !neg_pen && temp_ok;
  rc.decr = rc.fast && (!n.ctx || rc.rep >= 1.0f);
  return rc;
}

__device__ __forceinline__ float penalize(float v, bool seen, const RowConsts& rc) {
  if (!seen) return v;
  if (v < 0.0f) return __fmul_rn(v, rc.rep);
  return rc.rep_fast ? __fmul_rn(v, rc.rrep) : __fdiv_rn(v, rc.rep);
}

// The reference logit processors for two adjacent logits (ops/prologue.py:29-114, 443-447),
// in its order, rounding to bf16 after every operation. `g2` holds the two grammar bits.
__device__ __forceinline__ uint32_t process_pair(uint32_t x, uint32_t g2, int32_t d0, int32_t d1, int32_t c0,
                                                 int32_t c1, uint32_t b2, const RowConsts& rc) {
  if (rc.nd.proc) {
    if (rc.nd.g) {
      const uint32_t keep = ((g2 & 1u) ? 0x0000ffffu : 0u) | ((g2 & 2u) ? 0xffff0000u : 0u);
      x = (x & keep) | (0xff80ff80u & ~keep);
    }
    if (rc.nd.dec) {
      if (rc.nd.ctx) {
        const float lo = penalize(bf2_lo(x), d0 + c0 > 0, rc);
        const float hi = penalize(bf2_hi(x), d1 + c1 > 0, rc);
        x = bf2_pack(lo, hi);
      }
      if (rc.ind & 0x4) x = bf2_sub(x, bf2_mul(bf2_pack(__int2float_rn(d0), __int2float_rn(d1)), rc.freq2));
      if (rc.ind & 0x8) {
        // (decode > 0) * presence: the penalty itself, or a zero carrying its sign
        const uint32_t sel = ((d0 > 0) ? (rc.pres2 & 0x0000ffffu) : (rc.pres2 & 0x00008000u)) |
                             ((d1 > 0) ? (rc.pres2 & 0xffff0000u) : (rc.pres2 & 0x80000000u));
        x = bf2_sub(x, sel);
      }
    }
    if (rc.nd.bias) x = bf2_add(x, b2);
  }
  if (rc.nd.temp) {
    float lo = bf2_lo(x), hi = bf2_hi(x);
    if (rc.temp_fast) {
      lo = __fmul_rn(lo, rc.rtemp);
      hi = __fmul_rn(hi, rc.rtemp);
    } else {
      lo = __fdiv_rn(lo, rc.temp);
      hi = __fdiv_rn(hi, rc.temp);
    }
    x = bf2_pack(lo, hi);
  }
  return x;
}

// Raw inputs of 8 consecutive columns.
struct Raw8 {
  uint32_t x[4];   // bf16 pairs
  int32_t d[VPT];  // decode counts
  int32_t c[VPT];  // context counts
  uint32_t b[4];   // bias pairs
  uint32_t g;      // grammar bits (bit j = column j)
};

__device__ __forceinline__ void process8(Raw8& r, const RowConsts& rc) {
#pragma unroll
  for (int p = 0; p < 4; ++p)
    r.x[p] = process_pair(r.x[p], (r.g >> (2 * p)) & 3u, r.d[2 * p], r.d[2 * p + 1], r.c[2 * p], r.c[2 * p + 1],
                          r.b[p], rc);
}

// ---------------------------------------------------------------------------------------
// fast path of stochastic rows: penalties only where a count is nonzero (they are the
// identity elsewhere), temperature only for candidates (it is monotone, so the candidate
// test runs against the pre-temperature cut `vmin`), grammar as a mask bit
// ---------------------------------------------------------------------------------------

// final (post-temperature) value of a post-bias logit
__device__ __forceinline__ float temper(float v, bool on, bool fast, float t, float rt) {
  if (!on) return v;
  return rbf(fast ? __fmul_rn(v, rt) : __fdiv_rn(v, t));
}

__device__ __forceinline__ float final_value(float v, const RowConsts& rc) {
  return temper(v, rc.nd.temp, rc.temp_fast, rc.temp, rc.rtemp);
}

// multiplicative, frequency and presence penalties of one logit (ops/prologue.py:57-102)
__device__ __forceinline__ uint32_t repetition_one(uint32_t h, int32_t d, int32_t c, const RowConsts& rc) {
  float v = bf2f((uint16_t)h);
  if (rc.nd.ctx) v = rbf(penalize(v, d + c > 0, rc));
  if (rc.ind & 0x4) v = rbf(__fsub_rn(v, rbf(__fmul_rn(rbf(__int2float_rn(d)), bf2f((uint16_t)(rc.freq2 & 0xffffu))))));
  if (rc.ind & 0x8) v = rbf(__fsub_rn(v, bf2f((uint16_t)((d > 0) ? (rc.pres2 & 0xffffu) : (rc.pres2 & 0x8000u)))));
  return f2bf(v);
}

// 8-bit mask of the bf16 logits of x[0..3] that are >= the pair v2 (NaN never passes)
__device__ __forceinline__ uint32_t ge_mask8(const uint32_t (&x)[4], uint32_t v2) {
  uint32_t bits = 0;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t m = __hge2_mask(*reinterpret_cast<const __nv_bfloat162*>(&x[p]),
                                   *reinterpret_cast<const __nv_bfloat162*>(&v2));
    bits |= (m & 0x00010001u) << (2 * p);
  }
  return (bits | (bits >> 15)) & 0xffu;
}

__device__ __forceinline__ uint32_t ge_mask4(const uint32_t (&x)[2], uint32_t v2) {
  uint32_t bits = 0;
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const uint32_t m = __hge2_mask(*reinterpret_cast<const __nv_bfloat162*>(&x[p]),
                                   *reinterpret_cast<const __nv_bfloat162*>(&v2));
    bits |= (m & 0x00010001u) << (2 * p);
  }
  return (bits | (bits >> 15)) & 0xfu;
}

__device__ __forceinline__ uint32_t half_of(const uint32_t* x, int j) {
  return (j & 1) ? (x[j >> 1] >> 16) : (x[j >> 1] & 0xffffu);
}

// Greedy order key (ops/prologue.py:117-138 + ops/singular.py:71-131): value, then the
// lowest offset inside its block_n tile, then the lowest tile. -0.0 compares as +0.0.
__device__ __forceinline__ uint64_t greedy_key_bits(uint32_t h, int64_t c, int log2bn) {
  if (h == 0x8000u) h = 0;
  const uint64_t e = enc16(h);
  const int64_t bn = 1ll << log2bn;
  const uint64_t loc = (uint64_t)(bn - 1 - (c & (bn - 1)));
  const uint64_t tile = 0xffffffffull - (uint64_t)(c >> log2bn);
  return (e << 48) | (loc << 32) | tile;
}

__device__ __forceinline__ int64_t greedy_col(uint64_t key, int log2bn) {
  const int64_t tile = (int64_t)(0xffffffffu - (uint32_t)key);
  const int64_t loc = ((1ll << log2bn) - 1) - (int64_t)((key >> 32) & 0xffffu);
  return (tile << log2bn) + loc;
}

// ---------------------------------------------------------------------------------------
// direct (non-bulk) loads of 8 columns: vector loads when aligned, else scalar / gathered
// ---------------------------------------------------------------------------------------

template <int MODE>
__device__ __forceinline__ void load_x8(const uint16_t* xrow, int64_t c, int nvalid, uint32_t (&x)[4]) {
  if (MODE != kScalar && nvalid == VPT) {
    const uint4 q = ld_stream(xrow + c);
    x[0] = q.x;
    x[1] = q.y;
    x[2] = q.z;
    x[3] = q.w;
  } else {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t lo = (2 * p < nvalid) ? (uint32_t)__ldcs(xrow + c + 2 * p) : 0xff80u;
      const uint32_t hi = (2 * p + 1 < nvalid) ? (uint32_t)__ldcs(xrow + c + 2 * p + 1) : 0xff80u;
      x[p] = lo | (hi << 16);
    }
  }
}

// Aux values of 8 columns; `col[j]` are the aux-buffer columns (shard offset / d2t applied).
template <int MODE>
__device__ __forceinline__ void load_aux8(const SonicSamplingParams& P, const RowConsts& rc, int64_t slot,
                                          const int64_t (&col)[VPT], int nvalid, Raw8& r) {
  if (MODE != kScalar && nvalid == VPT) {
    if (rc.nd.dec) {
      const int32_t* d = P.decode_counts + slot * P.counts_stride + col[0];
      const uint4 p = ld_stream(d), q = ld_stream(d + 4);
      r.d[0] = p.x; r.d[1] = p.y; r.d[2] = p.z; r.d[3] = p.w;
      r.d[4] = q.x; r.d[5] = q.y; r.d[6] = q.z; r.d[7] = q.w;
    }
    if (rc.nd.ctx) {
      const int32_t* d = P.context_counts + slot * P.counts_stride + col[0];
      const uint4 p = ld_stream(d), q = ld_stream(d + 4);
      r.c[0] = p.x; r.c[1] = p.y; r.c[2] = p.z; r.c[3] = p.w;
      r.c[4] = q.x; r.c[5] = q.y; r.c[6] = q.z; r.c[7] = q.w;
    }
    if (rc.nd.bias) {
      const uint4 q = ld_stream(P.bias + slot * P.bias_stride + col[0]);
      r.b[0] = q.x; r.b[1] = q.y; r.b[2] = q.z; r.b[3] = q.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const bool ok = j < nvalid;
      r.d[j] = (rc.nd.dec && ok) ? __ldcs(P.decode_counts + slot * P.counts_stride + col[j]) : 0;
      r.c[j] = (rc.nd.ctx && ok) ? __ldcs(P.context_counts + slot * P.counts_stride + col[j]) : 0;
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const bool lo_ok = rc.nd.bias && 2 * p < nvalid, hi_ok = rc.nd.bias && 2 * p + 1 < nvalid;
      const uint32_t lo = lo_ok ? (uint32_t)__ldcs(P.bias + slot * P.bias_stride + col[2 * p]) : 0u;
      const uint32_t hi = hi_ok ? (uint32_t)__ldcs(P.bias + slot * P.bias_stride + col[2 * p + 1]) : 0u;
      r.b[p] = lo | (hi << 16);
    }
  }
}

template <int MODE>
__device__ __forceinline__ uint32_t load_g8(const SonicSamplingParams& P, int64_t grow, const int64_t (&col)[VPT],
                                            int nvalid) {
  const uint32_t* g = P.grammar + grow * P.grammar_stride;
  if (MODE != kScalar && nvalid == VPT) return (__ldg(g + (col[0] >> 5)) >> (col[0] & 31)) & 0xffu;
  uint32_t bits = 0;
#pragma unroll
  for (int j = 0; j < VPT; ++j)
    if (j < nvalid) bits |= ((__ldg(g + (col[j] >> 5)) >> (col[j] & 31)) & 1u) << j;
  return bits;
}

// ---------------------------------------------------------------------------------------
// candidate keys, tickets, list merges and the 128-wide selection steps
// ---------------------------------------------------------------------------------------

template <typename K>
__device__ __forceinline__ float key_value(K k);
template <>
__device__ __forceinline__ float key_value<uint32_t>(uint32_t k) { return bf2f(dec16(k >> 16)); }
template <>
__device__ __forceinline__ float key_value<uint64_t>(uint64_t k) { return dec32((uint32_t)(k >> 32)); }

// local key -> global sortable key ((enc << 32) | ~column); 0 for an empty slot
template <typename K>
__device__ __forceinline__ uint64_t to_global(K k, int64_t c0);
template <>
__device__ __forceinline__ uint64_t to_global<uint32_t>(uint32_t k, int64_t c0) {
  if (k == 0) return 0;
  const int64_t col = c0 + (0xffff - (int64_t)(k & 0xffffu));
  return ((uint64_t)(k >> 16) << 32) | (uint64_t)(0xffffffffu - (uint32_t)col);
}
template <>
__device__ __forceinline__ uint64_t to_global<uint64_t>(uint64_t k, int64_t c0) {
  if (k == 0) return 0;
  const int64_t col = c0 + (int64_t)(0xffffffffu - (uint32_t)k);
  return (k & 0xffffffff00000000ull) | (uint64_t)(0xffffffffu - (uint32_t)col);
}

// Ticket: true in the last CTA of the unit to arrive; that CTA also re-arms the ticket. A CTA
// that took the bounded-wait error path arrives with `failed`: the low 16 bits count the
// arrivals, the high 16 the failed ones, and `*row_failed` tells the last CTA whether any CTA
// of the unit failed (its outputs are then left unwritten).
__device__ __forceinline__ bool arrive_last(uint32_t* ticket, int splits, int* flag, bool failed = false,
                                            bool* row_failed = nullptr) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(ticket, failed ? 0x10001u : 1u);
    const bool last = (prev & 0xffffu) == (uint32_t)(splits - 1);
    if (last) *ticket = 0;
    *flag = (last ? 1 : 0) | ((failed || (prev >> 16)) ? 2 : 0);
  }
  __syncthreads();
  const int f = *flag;
  if (row_failed) *row_failed = (f & 2) != 0;
  const bool last = (f & 1) != 0;
  if (last) __threadfence();
  return last;
}

// Fold `splits` sorted candidate lists (u64 keys, descending) into one (warp-wide).
__device__ __forceinline__ void warp_fold_lists(const uint64_t* lists, int splits, int lane, uint64_t (&acc)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] = ldcg64(lists + 4 * lane + j);
  for (int s = 1; s < splits; ++s) {
    uint64_t b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) b[j] = ldcg64(lists + (int64_t)s * kMaxK + 4 * lane + j);
    warp_merge128_desc(acc, b, lane);
  }
}

__device__ __forceinline__ void decode_keys(const uint64_t (&k)[4], float (&v)[4], int64_t (&idx)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = bf2f(dec16((uint32_t)(k[j] >> 32)));
    idx[j] = (int64_t)(0xffffffffu - (uint32_t)k[j]);
  }
}

// Per-slot masking parameters, loaded early so the selection epilogue does not wait on them.
struct MaskParams {
  int32_t top_k, top_logprobs;
  uint16_t top_p, min_p;
  float log_min_p;  // log(min_p), computed once with the parameters
  bool has_k, has_p, has_min_p;
};

__device__ __forceinline__ MaskParams load_mask_params(const SonicSamplingParams& P, int64_t slot) {
  MaskParams m;
  m.has_k = P.top_k != nullptr;
  m.has_p = P.top_p != nullptr;
  m.has_min_p = P.min_p != nullptr;
  m.top_k = m.has_k ? P.top_k[slot] : 0;
  m.top_p = m.has_p ? P.top_p[slot] : 0;
  m.min_p = m.has_min_p ? P.min_p[slot] : 0;
  m.top_logprobs = P.top_logprobs ? P.top_logprobs[slot] : 0;
  m.log_min_p = m.has_min_p ? dlog(bf2f(m.min_p)) : 0.0f;
  return m;
}

__device__ __forceinline__ MaskParams mask_params(const SonicSamplingParams& P, const SlotScalars& s) {
  MaskParams m;
  m.has_k = P.top_k != nullptr;
  m.has_p = P.top_p != nullptr;
  m.has_min_p = P.min_p != nullptr;
  m.top_k = s.top_k;
  m.top_p = s.top_p;
  m.min_p = s.min_p;
  m.top_logprobs = s.top_logprobs;
  m.log_min_p = m.has_min_p ? dlog(bf2f(m.min_p)) : 0.0f;
  return m;
}

// cumulative_masking (ops/base.py:95-129) on the sorted top-128 held 4 per lane. When top-p
// runs, e receives exp(v - maximum) of the values it saw and the call returns true.
__device__ __forceinline__ bool warp_masking(const MaskParams& M, uint32_t ind, float (&v)[4], float maximum,
                                             int lane, float (&e)[4]) {
  const float ninf = __int_as_float(0xff800000);
  bool have_e = false;
  if ((ind & 0x80) && M.has_k) {
    const int32_t k = M.top_k;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(4 * lane + j < k)) v[j] = ninf;
  }
  if ((ind & 0x100) && M.has_p) {
    float lad[4];
    have_e = true;
#pragma unroll
    for (int j = 0; j < 4; ++j) e[j] = dexp(__fsub_rn(v[j], maximum));
    warp_ladder128(e, lad, lane);
    // ops/base.py:81-84 scales the prefix sum's last element, which is also the maximum of the
    // reference's never-decreasing prefix sums; this scan can end an ulp below an earlier prefix
    // past the last nonzero term (the lane totals are grouped differently), so take the maximum
    float total = fmaxf(fmaxf(lad[0], lad[1]), fmaxf(lad[2], lad[3]));
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) total = fmaxf(total, __shfl_xor_sync(kFull, total, d));
    const float scale = __fmul_rn(total, bf2f(M.top_p));
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(lad[j] <= scale || (lane == 0 && j == 0))) v[j] = ninf;
  }
  if ((ind & 0x200) && M.has_min_p) {
    const float pivot = __fadd_rn(M.log_min_p, maximum);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(v[j] >= pivot)) v[j] = ninf;
  }
  return have_e;
}

// log_softmax (ops/base.py:66-72) of 128 values held 4 per lane. With have_e, e already
// holds exp(v - maximum) for every value that is not -inf (from the top-p mask); it is
// reused instead of recomputed (exp(-inf) is 0, the same bits as recomputing).
__device__ __forceinline__ void warp_log_softmax(const float (&v)[4], float maximum, float (&ls)[4],
                                                 bool have_e = false, const float* e_in = nullptr) {
  float sc[4], e[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sc[j] = __fsub_rn(v[j], maximum);
    e[j] = have_e ? (v[j] == __int_as_float(0xff800000) ? 0.0f : e_in[j]) : dexp(sc[j]);
  }
  const float lse = dlog(warp_sum128(e));
#pragma unroll
  for (int j = 0; j < 4; ++j) ls[j] = __fsub_rn(sc[j], lse);
}

constexpr float kFiniteFloor = -3.40282346638528859811704183484516925e+38f;  // -FLT_MAX

// ---------------------------------------------------------------------------------------
// per-warp streaming top-128 of the single-row kernels
// ---------------------------------------------------------------------------------------
//
// Each warp keeps the 128 largest keys it has seen, sorted, in registers (4 per lane), plus a
// shared-memory queue of new keys at or above the CTA's cut. When 128 or more keys are
// queued the warp sorts them in blocks of 128 and merges each block into its list: no
// block-wide synchronisation. The cut is the largest 128th-kept-key value of any warp (128
// keys of the split are at least that large, so nothing below it can be in the split's
// top-128); it lives in shared memory as (enc32(value) << 32) | fast-path pre-temperature
// pair, both monotone in the value, so one 64-bit atomicMax publishes it. At the end of a
// split warp 0 merges the 8 lists.

constexpr int NW = NT / 32;
constexpr int QCAP = kMaxK + VPT * 32;  // a warp appends at most 256 keys per chunk
// singular_kernel's queue: 104 keys plus one group's 256, so that two CTAs with a 4-stage
// ring fit an SM's shared memory; a warp absorbs once more than SABSORB keys are queued
constexpr int SQCAP = 360;
constexpr int SABSORB = SQCAP - VPT * 32;

// ---------------------------------------------------------------------------------------
// Phase stamps: a diagnostic build only (-DSONIC_PHASE_STAMPS, `python -m
// sonic_sampler_b200.phases`). Each CTA of the singular kernels records %globaltimer (ns)
// at its phase boundaries, and each warp its clock cycles per activity, into a fixed device
// array that sonic_phase_stamps() copies out. In the product build every hook below is empty
// and compiles away.
// ---------------------------------------------------------------------------------------

enum PhaseCta {  // per-CTA %globaltimer stamps
  PS_ENTRY, PS_PDL, PS_SETUP, PS_FIRST, PS_WARP0_END, PS_ALL_END, PS_FOLD, PS_LIST, PS_TICKET, PS_MERGE,
  PS_SELECT, PS_SMID, PS_SCALARS, PS_ISSUED, PS_CTA_SLOTS
};
enum PhaseWarp {  // per-warp accumulated clock cycles / counts
  PW_WAIT, PW_PROCESS, PW_ABSORB, PW_ABSORBS, PW_PUSHED, PW_RELEASE, PW_END, PW_GROUPS, PW_PUSHPATH, PW_LOADS,
  PW_SLOTS
};
#ifdef SONIC_PHASE_STAMPS
constexpr int PS_CTAS = 8192;
struct PhaseStamps {
  unsigned long long cta[PS_CTAS][PS_CTA_SLOTS];
  unsigned long long warp[PS_CTAS][NW][PW_SLOTS];
};
__device__ PhaseStamps g_phase;

__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct PhaseClock {
  unsigned long long acc[PW_SLOTS];
  int cta;
  __device__ __forceinline__ PhaseClock() : cta((int)(blockIdx.y * gridDim.x + blockIdx.x)) {
#pragma unroll
    for (int i = 0; i < PW_SLOTS; ++i) acc[i] = 0;
  }
  __device__ __forceinline__ long long now() const { return clock64(); }
  __device__ __forceinline__ void add(int slot, long long since) { acc[slot] += (unsigned long long)(clock64() - since); }
  __device__ __forceinline__ void count(int slot, unsigned long long n) { acc[slot] += n; }
  // one thread of the CTA stamps slot `slot`
  __device__ __forceinline__ void stamp(int slot, bool who) const {
    if (who && cta < PS_CTAS) {
      g_phase.cta[cta][slot] = gtimer();
      if (slot == PS_ENTRY) {
        unsigned smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        g_phase.cta[cta][PS_SMID] = smid;
      }
    }
  }
  __device__ __forceinline__ void flush(int warp, int lane) {
    acc[PW_END] = gtimer();
    if (lane == 0 && cta < PS_CTAS)
      for (int i = 0; i < PW_SLOTS; ++i) g_phase.warp[cta][warp][i] = acc[i];
  }
};
#else
struct PhaseClock {
  __device__ __forceinline__ long long now() const { return 0; }
  __device__ __forceinline__ void add(int, long long) {}
  __device__ __forceinline__ void count(int, unsigned long long) {}
  __device__ __forceinline__ void stamp(int, bool) const {}
  __device__ __forceinline__ void flush(int, int) {}
};
#endif

template <typename K>
struct WarpTopK {
  K* list;         // shared memory, 128 keys sorted descending
  int qn;          // queued keys (warp-uniform)
  float thr;       // candidate threshold, final-value domain (warp-uniform)
  uint32_t vmin2;  // fast path: pre-temperature threshold pair (warp-uniform)
  unsigned long long cut;  // packed (thr, vmin2), see pack_cut
};

__device__ __forceinline__ unsigned long long pack_cut(float thr, uint32_t vmin2) {
  return ((unsigned long long)enc32(thr) << 32) | vmin2;
}

template <typename K>
__device__ __forceinline__ void wtk_init(WarpTopK<K>& w, K* list, float thr0, int lane) {
  w.list = list;
#pragma unroll
  for (int j = 0; j < 4; ++j) list[4 * lane + j] = 0;
  __syncwarp();
  w.qn = 0;
  w.thr = thr0;
  w.vmin2 = 0;
  w.cut = pack_cut(thr0, 0);
}

// take the CTA's cut when another warp raised it
template <typename K>
__device__ __forceinline__ void wtk_adopt(WarpTopK<K>& w, const unsigned long long* cut, int lane) {
  unsigned long long c = 0;
  if (lane == 0) c = *reinterpret_cast<const volatile unsigned long long*>(cut);
  c = __shfl_sync(kFull, c, 0);
  if (c > w.cut) {
    w.cut = c;
    w.thr = dec32((uint32_t)(c >> 32));
    w.vmin2 = (uint32_t)c;
  }
}

// raise this warp's threshold to `t` (with its fast-path pair `vm`) and publish it
template <typename K>
__device__ __forceinline__ void wtk_raise(WarpTopK<K>& w, unsigned long long* cut, float t, uint32_t vm, int lane) {
  w.thr = t;
  w.vmin2 = vm;
  w.cut = pack_cut(t, vm);
  if (lane == 0) atomicMax(cut, w.cut);
}

// warp-exclusive offsets of `np` items per lane; returns the warp total
__device__ __forceinline__ int warp_offsets(int np, int lane, int& excl) {
  int incl = np;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(kFull, incl, d);
    if (lane >= d) incl += y;
  }
  excl = incl - np;
  return __shfl_sync(kFull, incl, 31);
}

// append the keys of the set bits of `m` to the warp queue
template <typename K>
__device__ __forceinline__ void wtk_push(WarpTopK<K>& w, K* q, const K (&key)[VPT], unsigned m, int lane) {
  if (!__any_sync(kFull, m)) return;
  int excl;
  const int total = warp_offsets(__popc(m), lane, excl);
  int pos = w.qn + excl;
#pragma unroll
  for (int j = 0; j < VPT; ++j)
    if ((m >> j) & 1u) q[pos++] = key[j];
  w.qn += total;
}

// Sort the `qn` queued keys in blocks of 128 and merge each block into the warp's sorted
// list (both in shared memory); returns the value of the 128th kept key (-inf while fewer
// than 128 are kept). Not inlined: it runs rarely and is large, and one copy keeps the
// streaming loop inside the instruction cache.
// A non-zero `tq` marks queues that hold pre-temperature keys (the fast path of stochastic
// rows): their values are tempered (temper(v, 1, tfast, t, rt)) before the sort, so the list
// holds final keys and ties between final values fall back to the lowest column.
template <typename K>
__device__ __noinline__ float absorb_queue(K* list, const K* q, int qn, int lane, int tq, int tfast, float t,
                                           float rt, int kth) {
  __syncwarp();
  K l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) l[j] = list[4 * lane + j];
  for (int base = 0; base < qn; base += kMaxK) {
    K k[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = base + 4 * lane + j;
      k[j] = i < qn ? q[i] : (K)0;
      if (sizeof(K) == 4 && tq && k[j]) {
        const uint32_t u = (uint32_t)k[j];
        const float f = temper(bf2f((uint16_t)dec16(u >> 16)), true, tfast != 0, t, rt);
        k[j] = (K)((enc16(f2bf(f)) << 16) | (u & 0xffffu));
      }
    }
    warp_sort128_desc(k, lane);
    warp_merge128_desc(l, k, lane);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) list[4 * lane + j] = l[j];
  __syncwarp();
  // the kth kept key (kth = 128 unless only the first kth candidates can ever be selected)
  const int src = (kth - 1) >> 2, jj = (kth - 1) & 3;
  const K c0 = __shfl_sync(kFull, l[0], src), c1 = __shfl_sync(kFull, l[1], src);
  const K c2 = __shfl_sync(kFull, l[2], src), c3 = __shfl_sync(kFull, l[3], src);
  const K last = jj == 0 ? c0 : (jj == 1 ? c1 : (jj == 2 ? c2 : c3));
  return last != 0 ? key_value<K>(last) : __int_as_float(0xff800000);
}

template <typename K>
__device__ __forceinline__ float wtk_absorb(WarpTopK<K>& w, const K* q, int lane, bool tq = false,
                                            bool tfast = false, float t = 1.0f, float rt = 1.0f, int kth = kMaxK) {
  const float r = absorb_queue<K>(w.list, q, w.qn, lane, tq, tfast, t, rt, kth);
  w.qn = 0;
  return r;
}

// Merge the NW warp lists (shared memory, overwritten) into warp 0's registers with a
// 3-round tree. Block-wide.
template <typename K>
__device__ void block_fold(K (*lists)[kMaxK], int warp, int lane, K (&out)[4]) {
  __syncthreads();
#pragma unroll
  for (int width = NW / 2; width >= 1; width >>= 1) {
    if (warp < width) {
      K b[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        out[j] = lists[warp][4 * lane + j];
        b[j] = lists[warp + width][4 * lane + j];
      }
      warp_merge128_desc(out, b, lane);
      if (width > 1)
#pragma unroll
        for (int j = 0; j < 4; ++j) lists[warp][4 * lane + j] = out[j];
    }
    __syncthreads();
  }
}

__device__ __forceinline__ int64_t key_column(uint64_t g) { return (int64_t)(0xffffffffu - (uint32_t)g); }

// Merge `splits` sorted candidate lists of 128 u64 keys (workspace) into warp 0's registers.
// Warp v folds lists v, v+8, ... (all its loads issued at once), then a 3-round tree over
// shared memory (`xchg`, NW x 128 u64) combines the warp results. Block-wide.
__device__ void block_merge_lists(const uint64_t* lists, int splits, uint64_t* xchg, int warp, int lane,
                                  uint64_t (&out)[4], int64_t list_stride = kMaxK) {
  uint64_t acc[4] = {0, 0, 0, 0};
  if (warp < splits) {
    constexpr int PER = MAX_SPLITS / NW;
    uint64_t pre[PER][4];
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      const int s = warp + t * NW;
#pragma unroll
      for (int j = 0; j < 4; ++j) pre[t][j] = s < splits ? ldcg64(lists + (int64_t)s * list_stride + 4 * lane + j) : 0ull;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[j] = pre[0][j];
#pragma unroll
    for (int t = 1; t < PER; ++t)
      if (warp + t * NW < splits) warp_merge128_desc(acc, pre[t], lane);
  }
  // tree over the warps that hold lists (splits is uniform over the CTA)
  int width = 1;
  while (2 * width < min(splits, NW)) width *= 2;
  for (; width >= 1 && splits > 1; width >>= 1) {
    if (warp >= width && warp < 2 * width)
#pragma unroll
      for (int j = 0; j < 4; ++j) xchg[(warp - width) * kMaxK + 4 * lane + j] = acc[j];
    __syncthreads();
    if (warp < width) {
      uint64_t b[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = xchg[warp * kMaxK + 4 * lane + j];
      warp_merge128_desc(acc, b, lane);
    }
    if (width > 1) __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) out[j] = acc[j];
}

// ---------------------------------------------------------------------------------------
// single-row streaming: groups of 256 columns (8 per lane) owned by one warp each. Full
// 2048-column chunks of a split arrive through a CTA-wide ring of bulk-copy stages (one
// chunk, 5 large copies, per stage); warp w consumes the w-th 256 columns of each chunk and
// the last warp to finish a stage refills it, so warps never wait for one another within
// the ring's depth. Groups the ring cannot take (a ragged tail, unaligned or gathered rows)
// use direct loads.
// ---------------------------------------------------------------------------------------

constexpr int GROUP = VPT * 32;  // columns of one warp group
constexpr int PF_GROUPS = 4;     // L2 prefetch distance of direct loads, in groups of one warp
// bytes of one 2048-column chunk with every stream: logits, decode counts, context counts, bias
// (2 + 4 + 4 + 2 bytes a column) and grammar words
constexpr int SG_STAGE = CH * 12 + CH / 8;     // 24832
constexpr int RING_BYTES = STAGES * SG_STAGE;  // the ring's shared memory
constexpr int MAX_RING_STAGES = 16;            // stages of rows with fewer streams (logits only: 16)

// A ring wait: polls stage barrier `bar` for phase `parity`, and every 32 polls the CTA's
// abort flag, which a warp sets when one of its waits gave up. Returns false on a timeout
// (WAIT_LIMIT polls) or an abort; the caller then leaves the streaming loop.
__device__ __forceinline__ bool ring_wait(uint64_t* bar, uint32_t parity, const int* abort_flag) {
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 31u && *reinterpret_cast<const volatile int*>(abort_flag)) return false;
  }
  return false;
}

// The error path of a ring kernel (one thread): wait, bounded, for the last copy issued into
// every stage, so that no bulk copy lands in shared memory after the CTA has left.
__device__ __forceinline__ void ring_drain(uint64_t* bars, const int* nissued, int nst) {
  for (int i = 0; i < nst; ++i)
    if (nissued[i] > 0) mbar_wait_bounded(&bars[i], (uint32_t)((nissued[i] - 1) & 1), WAIT_LIMIT);
}

// Diagnostics (SONIC_FLAG_DEBUG_STALL_RING): a wait that runs out. The barrier is initialised
// with one expected arrival that nothing ever makes, and the wait gives up after a few polls.
constexpr uint32_t STALL_TEST_LIMIT = 1u << 10;

__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Smallest bf16 v (finite or +inf, as a bf16 pair) whose final value is >= thr: a guess
// from thr * temperature, corrected a few steps along the order-preserving encoding (the
// final value is monotone in v); binary search when the guess is far off.
constexpr uint32_t kEncLo = 0x0080u, kEncHi = 0xff80u;  // enc of -max finite .. enc of +inf

__device__ __noinline__ uint32_t vmin_search(float thr, bool on, bool fast, float t, float rt) {
  uint32_t lo = kEncLo, hi = kEncHi;
  while (lo < hi) {
    const uint32_t mid = (lo + hi) >> 1;
    if (temper(bf2f((uint16_t)dec16(mid)), on, fast, t, rt) >= thr) hi = mid;
    else lo = mid + 1;
  }
  return lo;
}

__device__ __forceinline__ uint32_t vmin_pair(float thr, bool on, bool fast, float t, float rt) {
  auto ok = [&](uint32_t e) { return temper(bf2f((uint16_t)dec16(e)), on, fast, t, rt) >= thr; };
  const float guess = on ? __fmul_rn(thr, t) : thr;
  uint32_t e = umin(umax(enc16(f2bf(guess)), kEncLo), kEncHi);
  bool done = false;
  if (ok(e)) {
    for (int i = 0; i < 4 && !done; ++i) {
      if (e == kEncLo || !ok(e - 1)) done = true;
      else --e;
    }
  } else {
    for (int i = 0; i < 4 && !done; ++i) {
      if (e == kEncHi) break;
      ++e;
      if (ok(e)) done = true;
    }
  }
  if (!done) e = vmin_search(thr, on, fast, t, rt);
  const uint32_t h = dec16(e);
  return h | (h << 16);
}

__device__ __forceinline__ uint32_t vmin_pair(float thr, const RowConsts& rc) {
  return vmin_pair(thr, rc.nd.temp, rc.temp_fast, rc.temp, rc.rtemp);
}

// Floor of a greedy row whose only processor is its temperature: the smallest bf16 logit whose
// tempered value is at least tv (out of line: it runs only when a warp's best key rises).
__device__ __noinline__ float greedy_floor(float tv, bool fast, float t, float rt) {
  return bf2f((uint16_t)(vmin_pair(tv, true, fast, t, rt) & 0xffffu));
}

// How many leading candidates of a row can ever matter: with top-k (k < 128) set, positions
// >= k are masked to -inf before top-p, min-p, the softmax and the selection, so only the
// exact top-k is needed (and the cut may come from the k-th key), unless top-Z logprobs
// beyond k or the candidates' probabilities are written. Multistep rows keep 128 (their
// stage-2 buffers hold all 128 candidates).
__device__ __forceinline__ int needed_candidates(const SonicSingularArgs& a, const SlotScalars& s, bool ms) {
  const SonicSamplingParams& P = a.params;
  const uint32_t ind = s.ind;
  if (ms || !(ind & 0x80) || !P.top_k || (a.flags & SONIC_FLAG_PROBABILITIES)) return kMaxK;
  const int32_t k = s.top_k;
  if (k < 1 || k >= kMaxK) return kMaxK;
  int z = 0;
  if ((a.flags & SONIC_FLAG_LOGPROBS) && (ind & 0x400) && a.max_top_logprobs > 0 && P.top_logprobs)
    z = min(s.top_logprobs, a.max_top_logprobs);
  return max(k, min(z, kMaxK));
}

__device__ __forceinline__ int needed_candidates(const SonicSingularArgs& a, uint32_t ind, int64_t slot, bool ms) {
  const SonicSamplingParams& P = a.params;
  if (ms || !(ind & 0x80) || !P.top_k || (a.flags & SONIC_FLAG_PROBABILITIES)) return kMaxK;
  const int32_t k = P.top_k[slot];
  if (k < 1 || k >= kMaxK) return kMaxK;
  int z = 0;
  if ((a.flags & SONIC_FLAG_LOGPROBS) && (ind & 0x400) && a.max_top_logprobs > 0 && P.top_logprobs)
    z = min(P.top_logprobs[slot], a.max_top_logprobs);
  return max(k, min(z, kMaxK));
}

// Shared-memory state of a single-row CTA; QC is the queue capacity of a warp (at least 127
// plus the most keys a warp group can push).
template <typename K, int QC = QCAP>
struct RowSmem {
  K queue[NW][QC];
  K lists[NW][kMaxK];
  unsigned long long cut;  // packed CTA cut, see pack_cut
  int qn[NW];              // keys queued by each warp (singular_kernel: lanes reserve with atomics)
  float v16[NW];           // each warp's m-th kept key value (-inf while it keeps fewer)
  float vlm[NW];           // each warp's m-th largest lane maximum (see lane_max_publish)
  MaskParams mp;           // the slot's masking parameters (selection epilogue)
  int flag;
  unsigned long long best;
  int32_t toks[SONIC_MAX_LOOKAHEAD + 1];
  uint64_t bars[MAX_RING_STAGES];  // bulk-copy stage filled
  int rel[MAX_RING_STAGES];        // warps done with the stage
  int nissued[MAX_RING_STAGES];    // chunks issued into the stage (error-path drain)
  uint64_t stall_bar;              // diagnostics: a barrier nothing completes
  int abort;                       // a ring wait gave up: every warp leaves the streaming loop
};

// After an absorb: the warp's new threshold candidates are its own kk-th key value (own) and
// the smallest m-th key value over all warps (the 8 top-m sets are 8m >= kk distinct keys),
// kk the number of leading candidates the row needs exactly (128 unless top-k is smaller).
template <typename K>
__device__ __forceinline__ float absorbed_cut(const WarpTopK<K>& w, float own, float* v16, int warp, int lane,
                                             int m = 16) {
  const K km = w.list[m - 1];
  if (lane == 0) reinterpret_cast<volatile float*>(v16)[warp] = km ? key_value<K>(km) : __int_as_float(0xff800000);
  __syncwarp();
  float lo = lane < NW ? reinterpret_cast<volatile float*>(v16)[lane] : __int_as_float(0x7f800000);
#pragma unroll
  for (int d = 4; d >= 1; d >>= 1) lo = fminf(lo, __shfl_xor_sync(kFull, lo, d));
  lo = __shfl_sync(kFull, lo, 0);
  return fmaxf(own, lo);
}

// elementwise max of two bf16 pairs; a NaN loses to the other operand (IEEE maxNum)
__device__ __forceinline__ uint32_t bf2_max(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// descending bitonic sort of one value per lane
__device__ __forceinline__ uint32_t warp_sort32_desc(uint32_t v, int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int d = size >> 1; d >= 1; d >>= 1) {
      const uint32_t o = __shfl_xor_sync(kFull, v, d);
      const bool keep_max = ((lane & d) == 0) == ((lane & size) == 0 || size == 32);
      v = keep_max ? umax(v, o) : umin(v, o);
    }
  }
  return v;
}

// Each lane's largest key belongs to a distinct column, so the m-th largest lane maximum of
// every warp bounds 8m distinct keys of the split from below: with 8m >= kk (the leading
// candidates the row needs; m = 16 for all 128) the smallest of those over the warps is a
// valid cut. lane_max_publish stores a warp's m-th largest lane maximum (as a final value);
// lane_max_min reads the smallest over the warps.
template <typename F>
__device__ __forceinline__ void lane_max_publish(uint32_t lmax, float* vlm, int warp, int lane, F final_of,
                                                 int m = 16) {
  const uint32_t k16 = __shfl_sync(kFull, warp_sort32_desc(lmax, lane), m - 1);
  if (lane == 0)
    reinterpret_cast<volatile float*>(vlm)[warp] = k16 ? final_of(key_value<uint32_t>(k16)) : __int_as_float(0xff800000);
}

__device__ __forceinline__ float lane_max_min(const float* vlm, int lane) {
  float m = lane < NW ? reinterpret_cast<const volatile float*>(vlm)[lane] : __int_as_float(0x7f800000);
#pragma unroll
  for (int d = 4; d >= 1; d >>= 1) m = fminf(m, __shfl_xor_sync(kFull, m, d));
  return __shfl_sync(kFull, m, 0);
}

__device__ __forceinline__ uint32_t select4(const uint32_t (&v)[4], int i) {
  return i < 2 ? (i == 0 ? v[0] : v[1]) : (i == 2 ? v[2] : v[3]);
}

template <typename K, int QC>
__device__ __forceinline__ void row_smem_init(RowSmem<K, QC>& st, unsigned long long cut0) {
  st.cut = cut0;
  for (int i = 0; i < NW; ++i) st.v16[i] = st.vlm[i] = __int_as_float(0xff800000);
}

// Drafted tokens counted as decoded (ops/prologue.py:175-193) for columns whose aux values were
// gathered through a draft-to-target table: the drafted tokens are target ids, so they are
// matched against the columns' target ids `col` (the caller counts them by position otherwise).
__device__ __forceinline__ void add_drafted(Raw8& raw, const int64_t (&col)[VPT], int nvalid, const int32_t* toks,
                                            int ntok) {
  for (int t = 0; t < ntok; ++t) {
    const int64_t d = toks[t];
#pragma unroll
    for (int j = 0; j < VPT; ++j)
      if (j < nvalid) raw.d[j] += (col[j] == d);
  }
}

// Loads of one group of 8 columns per lane (`c` = first column of this lane). With a
// draft-to-target table (INDIRECT) the `ntok` drafted tokens `toks` are added to the decode
// counts here, by target id.
template <int MODE, bool INDIRECT>
__device__ __forceinline__ void load_group(const SonicSingularArgs& a, const RowConsts& rc, int64_t slot,
                                           int64_t gslot, const uint16_t* xrow, int64_t c, int nvalid, Raw8& raw,
                                           const int32_t* toks = nullptr, int ntok = 0) {
  constexpr int AM = INDIRECT ? kScalar : MODE;
  load_x8<MODE>(xrow, c, nvalid, raw.x);
  raw.g = 0xffu;
  if (rc.nd.proc) {
    int64_t col[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      col[j] = c + j + a.shard_offset;
      if (INDIRECT && j < nvalid) col[j] = load_index(a.d2t, a.d2t_dtype, col[j]);
    }
    load_aux8<AM>(a.params, rc, slot, col, nvalid, raw);
    if (rc.nd.g) raw.g = load_g8<AM>(a.params, gslot, col, nvalid);
    if (INDIRECT) add_drafted(raw, col, nvalid, toks, ntok);
  }
}

// Rows of a multistep call streamed by singular_kernel (MS mode): row r of the flattened
// logits is step s of request b; request b's steps are rows [margin, margin + T).
struct MsRows {
  const int32_t* cu_seqlens;  // varlen: [batch + 1] row offsets, else NULL (T = lookahead + 1)
  const int32_t* tokens;      // flattened drafted tokens [rows]
  int32_t batch;
  int32_t lookahead;
};

// request and step of multistep row r; false for a row outside every request
__device__ __forceinline__ bool ms_row(const MsRows& m, int64_t r, int64_t& b, int& s, int64_t& margin) {
  if (!m.cu_seqlens) {
    b = r / (m.lookahead + 1);
    s = (int)(r % (m.lookahead + 1));
    margin = b * (m.lookahead + 1);
    return b < m.batch;
  }
  int lo = 0, hi = m.batch;  // largest b with cu_seqlens[b] <= r
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (m.cu_seqlens[mid] <= r) lo = mid;
    else hi = mid;
  }
  b = lo;
  margin = m.cu_seqlens[lo];
  const int64_t t = m.cu_seqlens[lo + 1] - margin;
  s = (int)(r - margin);
  return r >= margin && s < t && s <= m.lookahead;
}

// ---------------------------------------------------------------------------------------
// selection epilogue of one row (ops/base.py:66-129, ops/singular.py:259-358) on its merged,
// sorted top-128 keys held 4 per lane by one warp
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ void select_row(const SonicSingularArgs& a, int64_t r, int64_t slot, uint32_t ind,
                                           const MaskParams& mp, const uint64_t (&k)[4], int lane) {
  const SonicSamplingParams& P = a.params;
  const uint32_t flags = a.flags;
  float v[4];
  int64_t idx[4];
  decode_keys(k, v, idx);
  // a column outside the row can only come from a workspace that was not zero-filled: such a
  // candidate is dropped instead of being gathered
  bool bad[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    bad[j] = idx[j] < 0 || idx[j] >= a.vocab_size;
    if (bad[j]) {
      v[j] = __int_as_float(0xff800000);
      idx[j] = 0;
    }
  }
  int64_t tok[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) tok[j] = a.d2t ? load_index(a.d2t, a.d2t_dtype, idx[j]) : idx[j];
  // noise loads first: their latency overlaps the masking
  uint16_t noise[4] = {0, 0, 0, 0};
  bool off[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    off[j] = bad[j] || (a.target_vocab > 0 && (tok[j] < 0 || tok[j] >= a.target_vocab));
    if (!(flags & SONIC_FLAG_PHILOX) && !off[j]) noise[j] = a.gumbel[slot * a.gumbel_stride + tok[j]];
  }
  const float vmax = __shfl_sync(kFull, v[0], 0);
  float ev[4];
  const bool have_e = (ind & 0x380) ? warp_masking(mp, ind, v, vmax, lane, ev) : false;
  float diff[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (flags & SONIC_FLAG_PHILOX)
      diff[j] = __fsub_rn(v[j], philox_log_exponential(a.philox_seed, a.philox_offset, (uint32_t)slot,
                                                        (uint32_t)tok[j]));
    else
      diff[j] = off[j] ? __int_as_float(0xff800000) : rbf(__fsub_rn(v[j], bf2f(noise[j])));
  }
  const int sel = warp_argmax128(diff, lane);
  const int64_t token = warp_pick128(tok, sel);
  if (lane == 0 && (flags & SONIC_FLAG_UPDATE_COUNTS) && token >= 0 && token < P.counts_stride) {
    int32_t* d = P.decode_counts + slot * P.counts_stride + token;
    if (flags & SONIC_FLAG_PREFILL) *d = 1;
    else atomicAdd(d, 1);
  }
  if (flags & (SONIC_FLAG_LOGPROBS | SONIC_FLAG_PROBABILITIES)) {
    float ls[4];
    warp_log_softmax(v, vmax, ls, have_e && vmax != __int_as_float(0xff800000), ev);
    if ((flags & SONIC_FLAG_LOGPROBS) && a.logprobs) {
      const float lsel = warp_pick128(ls, sel);
      if (lane == 0) store_float(a.logprobs, a.logprobs_dtype, r * a.logprobs_stride, lsel);
      if (a.max_top_logprobs > 0 && (ind & 0x400) && a.top_logprob_values && P.top_logprobs) {
        const int z = min(mp.top_logprobs, a.max_top_logprobs);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = 4 * lane + j;
          if (i < z) {
            store_float(a.top_logprob_values, a.logprobs_dtype, r * a.top_stride + i, ls[j]);
            a.top_logprob_tokens[r * a.top_stride + i] = (int32_t)tok[j];
          }
        }
      }
    }
    if ((flags & SONIC_FLAG_PROBABILITIES) && a.probabilities) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float p = dexp(ls[j]);
        if (!bad[j] && (a.target_vocab <= 0 || (tok[j] >= 0 && tok[j] < a.target_vocab)))
          store_float(a.probabilities, a.probabilities_dtype, slot * a.probabilities_stride + tok[j], p);
      }
    }
  }
  if (lane == 0) a.tokens[r * a.tokens_stride] = (int32_t)token;
}

// ---------------------------------------------------------------------------------------
// fused singular: prologue + top-128 per split + merge + selection
// (ops/prologue.py:272 + ops/singular.py:154)
// ---------------------------------------------------------------------------------------

// WIDE: a CTA covers more than 65536 columns (grids of several waves, one CTA per row): its
// warps' keys carry warp-local column indices and are folded as 64-bit global keys. Otherwise
// (cols <= 65536) the keys carry the CTA-local column and the fold runs on 32-bit keys.
template <int MODE, bool INDIRECT, bool MS, bool WIDE = false>
__global__ void __launch_bounds__(NT) singular_kernel(const SonicSingularArgs a, int splits, int cols, int log2bn,
                                                      Workspace ws, uint64_t* cand_out, const MsRows ms) {
  __shared__ __align__(16) RowSmem<uint32_t, SQCAP> st;
  extern __shared__ __align__(128) unsigned char smem_ring[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int64_t r = blockIdx.y;
  const SonicSamplingParams& P = a.params;
  const int64_t c0 = (int64_t)split * cols;
  const int64_t c1 = min((int64_t)a.vocab_size, c0 + cols);
  // The 16-bit column index of a key. WIDE: warp-local, column c0 + 2048 k + 256 w + i (warp
  // w's group in chunk k, i < 256) is (k << 8) | i, so a CTA covers up to 256 chunks
  // (SPLIT_MAX_COLS columns), and keys of different warps meet only as 64-bit keys with global
  // columns (the end-of-split fold). Else the CTA-local column c - c0 (< 65536).
  auto wloc = [&](int64_t c) {
    const uint32_t d = (uint32_t)(c - c0);
    return WIDE ? (((d >> 11) << 8) | (d & (GROUP - 1))) : d;
  };
  PhaseClock pc;
  pc.stamp(PS_ENTRY, tid == 0);

  pdl_wait();
  pc.stamp(PS_PDL, tid == 0);

  // Chunk 0's logits sit at offset 0 of stage 0 in every stage layout: that copy goes out
  // before the row's parameters are loaded (its bytes are expected without an arrival; the
  // arrival comes with the row's other streams, or on the way out).
  const uint16_t* xrow = (const uint16_t*)a.logits + r * a.logits_stride;
  const int nch = MODE == kTma ? (int)((c1 - c0) / CH) : 0;
  if (nch > 0 && tid == 0) {
    for (int i = 0; i < MAX_RING_STAGES; ++i) {
      mbar_init(&st.bars[i], 1);
      st.rel[i] = 0;
      st.nissued[i] = 0;
    }
    mbar_init(&st.stall_bar, 1);
    mbar_fence_init();
    mbar_expect_tx_only(&st.bars[0], CH * 2);
    bulk_load(smem_ring, xrow + c0, CH * 2, &st.bars[0]);
  }
  auto drain = [&]() {  // leaving early: the copy lands before the CTA does
    if (nch > 0 && tid == 0) {
      mbar_arrive(&st.bars[0]);
      mbar_wait_bounded(&st.bars[0], 0u, WAIT_LIMIT);
    }
  };

  // MS: row r is step `step` of multistep request `req` (rows [margin, margin + T))
  int64_t req = r, margin = 0;
  int step = 0;
  if (MS && !ms_row(ms, r, req, step, margin)) {
    drain();
    return;
  }
  const int64_t slot = load_slot(P, req);
  if (slot < 0 || (P.num_slots > 0 && slot >= P.num_slots)) {
    // out-of-range slot id: no CTA of this row touches per-slot buffers or the ticket
    if (!MS && split == 0 && tid == 0) a.tokens[r * a.tokens_stride] = -1;
    drain();
    return;
  }
  const SlotScalars sc = load_slot_scalars(P, slot);
  const uint32_t ind = sc.ind;
  const RowConsts rc = row_consts(P, sc);
  pc.stamp(PS_SCALARS, tid == 0);
  // vocab-sharded step 1 (cand_out) keeps greedy rows' candidates too: exact path, top-128
  const bool greedy = (ind & 0x40) != 0 && !cand_out;
  const int kk = needed_candidates(a, sc, MS);  // exact leading candidates needed
  const int mm = (kk + NW - 1) / NW;                   // of them per warp (cut rules)
  // drafted tokens counted as decoded: singular counts all `lookahead` drafted tokens of the
  // slot (ops/prologue.py:175-184); multistep step s counts the request's first s
  const int ntok = !rc.nd.dec ? 0 : (MS ? step : (a.drafted_tokens ? a.lookahead : 0));
  if (tid < ntok) st.toks[tid] = MS ? ms.tokens[margin + tid] : a.drafted_tokens[slot * a.drafted_stride + tid];
  // grammar row: per slot, or per (slot, step) in multistep (ops/prologue.py:29-54)
  const int64_t gslot = MS ? slot * (ms.lookahead + 1) + step : slot;
  // streams of the bulk-copy ring (see below)
  const int64_t shard = a.shard_offset;
  const uint32_t* grow = rc.nd.g ? P.grammar + gslot * P.grammar_stride : nullptr;
  const int32_t* drow = rc.nd.dec ? P.decode_counts + slot * P.counts_stride : nullptr;
  const int32_t* crow = rc.nd.ctx ? P.context_counts + slot * P.counts_stride : nullptr;
  const uint16_t* brow = rc.nd.bias ? P.bias + slot * P.bias_stride : nullptr;
  // stage layout of this row: only the streams it reads, as many stages as fit the ring. With a
  // draft-to-target table (INDIRECT) the ring carries the logits alone: the aux rows are
  // indexed by target id, so those values are gathered per group instead.
  const int32_t* rdrow = INDIRECT ? nullptr : drow;
  const int32_t* rcrow = INDIRECT ? nullptr : crow;
  const uint16_t* rbrow = INDIRECT ? nullptr : brow;
  const uint32_t* rgrow = INDIRECT ? nullptr : grow;
  const int sg_d = CH * 2;
  const int sg_c = sg_d + (rdrow ? CH * 4 : 0);
  const int sg_b = sg_c + (rcrow ? CH * 4 : 0);
  const int sg_g = sg_b + (rbrow ? CH * 2 : 0);
  const int sg_stage = sg_g + (rgrow ? CH / 8 : 0);  // bytes of one 2048-column chunk (multiple of 256)
  // Greedy rows without processors (a positive temperature at most) take 4096-column chunks
  // (8 KB) of logits: a warp then handles two adjacent groups per chunk, so the stage wait and
  // release are paid once per 512 columns of this almost free per-column work. Such a row
  // needs one full wide chunk (chunk 0's first half is already on its way).
  // Long CTAs take wider chunks still (WIDE_GROUPS_LONG groups a warp); short ones keep two,
  // which leaves fewer columns to the direct-load tail after the last full chunk.
  const int wg = (c1 - c0) >= WIDE_LONG_COLS ? WIDE_GROUPS_LONG : WIDE_GROUPS;
  const bool wide = MODE == kTma && (ind & 0x40) && !cand_out && !rc.nd.proc && sg_stage == CH * 2 &&
                    (!rc.nd.temp || (rc.temp > 0.0f && rc.temp <= 3.3895313892515355e+38f)) &&
                    (c1 - c0) >= wg * CH;
  const int cw = wide ? wg * CH : CH;                   // columns of a ring chunk
  const int stage_bytes = wide ? wg * CH * 2 : sg_stage;  // bytes of a ring stage
  const int nst = min(MAX_RING_STAGES, RING_BYTES / stage_bytes);
  const int nck = MODE == kTma ? (int)((c1 - c0) / cw) : 0;  // ring chunks of this split
  auto issue_chunk = [&](int i, int stage) {  // one thread
    unsigned char* sp = smem_ring + stage * stage_bytes;
    uint64_t* bar = &st.bars[stage];
    const int64_t cc = c0 + (int64_t)i * cw;
    ++st.nissued[stage];
    if (i == 0) {
      // the first 2048 columns' logits are on their way already
      if (wide) {
        mbar_expect_tx(bar, (uint32_t)((wg - 1) * CH * 2));
        bulk_load(sp + CH * 2, xrow + cc + CH, (uint32_t)((wg - 1) * CH * 2), bar);
      } else if (sg_stage > CH * 2) {
        mbar_expect_tx(bar, (uint32_t)(sg_stage - CH * 2));
      } else {
        mbar_arrive(bar);
      }
    } else {
      mbar_expect_tx(bar, (uint32_t)stage_bytes);
      bulk_load(sp, xrow + cc, cw * 2, bar);
    }
    if (rdrow) bulk_load(sp + sg_d, rdrow + cc + shard, CH * 4, bar);
    if (rcrow) bulk_load(sp + sg_c, rcrow + cc + shard, CH * 4, bar);
    if (rbrow) bulk_load(sp + sg_b, rbrow + cc + shard, CH * 2, bar);
    if (rgrow) bulk_load(sp + sg_g, rgrow + (cc + shard) / 32, CH / 8, bar);
  };
  if (tid < NW) st.qn[tid] = 0;
  if (tid == 0) {
    st.abort = 0;
    // stage 0's copies first: the stages land roughly in the order they are requested
    for (int i = 0; i < min(nck, nst); ++i) issue_chunk(i, i);  // barriers set up above
    pc.stamp(PS_ISSUED, true);
    st.best = 0ull;
    st.mp = mask_params(P, sc);
    row_smem_init(st, pack_cut(kFiniteFloor, rc.fast ? vmin_pair(kFiniteFloor, rc) : 0u));
  }
  __syncthreads();
  pc.stamp(PS_SETUP, tid == 0);
  bool werr = false;
  if ((a.flags & SONIC_FLAG_DEBUG_STALL_RING) && nck > 0) {
    // diagnostics: a wait that runs out, then the same error path as a real timeout
    if (!mbar_wait_bounded(&st.stall_bar, 0u, STALL_TEST_LIMIT)) werr = true;
    if (werr && lane == 0) *reinterpret_cast<volatile int*>(&st.abort) = 1;
  }

  uint32_t* q = st.queue[warp];
  WarpTopK<uint32_t> w;
  wtk_init(w, st.lists[warp], kFiniteFloor, lane);  // the first wtk_adopt takes the fast-path pair from st.cut
  uint64_t best = 0;
  // Greedy rows whose only processor is a temperature t in (0, max]: bf16(x / t) is monotone
  // in the logit x, so a column whose logit is below the warp's floor (the smallest bf16
  // whose tempered value reaches the best key the warp has seen) has a strictly smaller key
  // and is skipped with one compare; the others are tempered and keyed exactly.
  const bool gskip = greedy && !rc.nd.proc && rc.nd.temp && rc.temp > 0.0f && rc.temp <= 3.3895313892515355e+38f;
  float gfloor = __int_as_float(0xff800000);
  uint64_t gbest = 0;  // the warp's best key when gfloor was set
  bool tq = rc.fast && rc.nd.temp;  // fast-path queues hold pre-temperature keys
  auto final_of = [&](float v) { return final_value(v, rc); };

  // Queue slots: each lane with candidates reserves its slots with one shared-memory atomic on
  // the warp's counter (no warp-wide scan or vote); the queue order is immaterial, as absorbs
  // sort and keep the top of the union. `sync_qn` makes the count warp-uniform again.
  auto reserve = [&](int np) { return np ? atomicAdd(&st.qn[warp], np) : 0; };
  auto sync_qn = [&]() {
    __syncwarp();
    w.qn = *reinterpret_cast<volatile int*>(&st.qn[warp]);
  };
  auto absorb_if_full = [&]() {
    if (w.qn > SABSORB) {
      const long long ta = pc.now();
      const float t = absorbed_cut(w, wtk_absorb(w, q, lane, tq, rc.temp_fast, rc.temp, rc.rtemp, kk), st.v16, warp,
                                   lane, mm);
      if (lane == 0) st.qn[warp] = 0;
      __syncwarp();
      if (t > w.thr) wtk_raise(w, &st.cut, t, rc.fast ? vmin_pair(t, rc) : 0u, lane);
      pc.add(PW_ABSORB, ta);
      pc.count(PW_ABSORBS, 1);
    }
  };

  // exact path: every processor on every column, then the candidate test
  // greedy keys of a group of a row without processors: under the tempered-value floor
  // (gskip), else of the raw logits
  auto greedy_group = [&](const Raw8& raw, int64_t c, int nvalid) {
    if (!gskip) {
#pragma unroll
      for (int j = 0; j < VPT; ++j)
        if (j < nvalid) best = umax(best, greedy_key_bits(half_of(raw.x, j), c + j, log2bn));
      return;
    }
    bool rose = false;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float lo = bf2_lo(raw.x[p]), hi = bf2_hi(raw.x[p]);
      const bool e0 = 2 * p < nvalid && !(lo < gfloor);
      const bool e1 = 2 * p + 1 < nvalid && !(hi < gfloor);
      if (e0 || e1) {
        // the temperature step of process_pair, on this pair only
        const uint32_t tp = rc.temp_fast ? bf2_pack(__fmul_rn(lo, rc.rtemp), __fmul_rn(hi, rc.rtemp))
                                         : bf2_pack(__fdiv_rn(lo, rc.temp), __fdiv_rn(hi, rc.temp));
        const uint64_t k0 = e0 ? greedy_key_bits(tp & 0xffffu, c + 2 * p, log2bn) : 0ull;
        const uint64_t k1 = e1 ? greedy_key_bits(tp >> 16, c + 2 * p + 1, log2bn) : 0ull;
        const uint64_t k = umax(k0, k1);
        rose |= k > best;
        best = umax(best, k);
      }
    }
    // raise the warp's floor when its best key rose (warp-uniform; a NaN or -inf best
    // leaves the floor where it is, so ties and NaNs stay exact)
    if (__any_sync(kFull, rose)) {
      const uint64_t wb = warp_max_u64(best);
      if (wb > gbest) {
        gbest = wb;
        const float tv = bf2f((uint16_t)dec16((uint32_t)(wb >> 48)));
        if (tv > __int_as_float(0xff800000)) gfloor = greedy_floor(tv, rc.temp_fast, rc.temp, rc.rtemp);
      }
    }
  };

  auto exact_group = [&](Raw8& raw, int64_t c, int nvalid) {
    if (gskip) {
      greedy_group(raw, c, nvalid);
      return;
    }
    if (!INDIRECT && rc.nd.proc && ntok) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int64_t col = c + j + shard;
        for (int s = 0; s < ntok; ++s) raw.d[j] += (st.toks[s] == col);
      }
    }
    if (rc.nd.proc || rc.nd.temp) process8(raw, rc);
    if (greedy) {
#pragma unroll
      for (int j = 0; j < VPT; ++j)
        if (j < nvalid) best = umax(best, greedy_key_bits(half_of(raw.x, j), c + j, log2bn));
      return;
    }
    const float thr = w.thr;
    uint32_t key[VPT];
    unsigned m = 0;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const uint32_t h = half_of(raw.x, j);
      key[j] = (enc16(h) << 16) | (0xffffu - wloc(c + j));
      if (j < nvalid && bf2f((uint16_t)h) >= thr) m |= 1u << j;
    }
    int pos = reserve(__popc(m));
#pragma unroll
    for (int j = 0; j < VPT; ++j)
      if ((m >> j) & 1u) q[pos++] = key[j];
    sync_qn();
  };

  // fast path (see vmin_pair): temperature only for candidates, grammar as a mask bit, and
  // penalties only where a count is nonzero (they are the identity elsewhere). Where the
  // penalties cannot raise a logit (rc.decr, counts >= 0) the candidate test runs on the
  // unpenalised value first and only candidates are penalised and tested again.
  auto fast_group = [&](const Raw8& raw, int64_t c, int nvalid) -> int {
    uint32_t x[4] = {raw.x[0], raw.x[1], raw.x[2], raw.x[3]};
    // columns whose counts (or drafted tokens) are nonzero; computed only when needed
    auto need_bits = [&]() {
      uint32_t need = 0;
#pragma unroll
      for (int j = 0; j < VPT; ++j) need |= (uint32_t)((raw.d[j] | (rc.nd.ctx ? raw.c[j] : 0)) != 0) << j;
      for (int t = 0; t < (INDIRECT ? 0 : ntok); ++t) {
        const int64_t dl = (int64_t)st.toks[t] - (c + shard);
        if (dl >= 0 && dl < nvalid) need |= 1u << dl;
      }
      return need;
    };
    auto penalise = [&](uint32_t (&v)[4], uint32_t bits) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        if ((bits >> j) & 1u) {
          int32_t dj = raw.d[j];
          for (int t = 0; t < (INDIRECT ? 0 : ntok); ++t) dj += (st.toks[t] == c + j + shard);
          const uint32_t h = repetition_one(half_of(v, j), dj, rc.nd.ctx ? raw.c[j] : 0, rc);
          v[j >> 1] = (j & 1) ? ((v[j >> 1] & 0xffffu) | (h << 16)) : ((v[j >> 1] & 0xffff0000u) | h);
        }
      }
    };
    bool counted = ntok > 0;  // some count of this lane's columns may be nonzero
    if (rc.nd.dec) {
      int32_t any = 0;
#pragma unroll
      for (int j = 0; j < VPT; ++j) any |= raw.d[j] | (rc.nd.ctx ? raw.c[j] : 0);
      counted = counted || any != 0;
      // penalties that may raise a logit go in before the candidate test
      const bool before = counted && (!rc.decr || any < 0);
      if (__any_sync(kFull, before)) {
        if (before) penalise(x, need_bits());
        counted = counted && !before;
      }
    }
    uint32_t y[4] = {x[0], x[1], x[2], x[3]};
    if (rc.nd.bias) {
#pragma unroll
      for (int p = 0; p < 4; ++p) y[p] = bf2_add(x[p], raw.b[p]);
    }
    uint32_t m = ge_mask8(y, w.vmin2) & raw.g;
    if (nvalid < VPT) m &= (1u << max(nvalid, 0)) - 1u;
    if (m) {
      const long long tpp = pc.now();
      // candidates of the unpenalised test: penalise those with nonzero counts, test again
      if (counted) {
        const uint32_t late = m & need_bits();
        if (late) {
          penalise(x, late);
#pragma unroll
          for (int p = 0; p < 4; ++p) y[p] = rc.nd.bias ? bf2_add(x[p], raw.b[p]) : x[p];
          m &= ge_mask8(y, w.vmin2) | ~late;
        }
      }
      int pos = reserve(__popc(m));
      const uint32_t base = 0xffffu - wloc(c);
      pc.count(PW_PUSHED, (unsigned long long)__popc(m));
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1;
        const uint32_t word = select4(y, j >> 1);
        q[pos++] = (enc16((j & 1) ? (word >> 16) : (word & 0xffffu)) << 16) | (base - (uint32_t)j);
      }
      pc.add(PW_PUSHPATH, tpp);
    }
    sync_qn();
    return 0;
  };

  auto process_group = [&](Raw8& raw, int64_t c, int nvalid, int k) {
    const long long tp = pc.now();
    if (!greedy) wtk_adopt(w, &st.cut, lane);
    if (rc.fast)
      fast_group(raw, c, nvalid);
    else
      exact_group(raw, c, nvalid);
    if (!greedy) absorb_if_full();
    pc.add(PW_PROCESS, tp);
    pc.count(PW_GROUPS, 1);
  };

  // groups of this warp: g = warp, warp + NW, ...; columns [c0 + g * GROUP, +GROUP)
  const int ngroups = (int)((c1 - c0 + GROUP - 1) / GROUP);
  auto gcol = [&](int g) { return c0 + (int64_t)g * GROUP + (int64_t)VPT * lane; };
  auto gvalid = [&](int g) { return (int)max((int64_t)0, min((int64_t)VPT, c1 - gcol(g))); };
  constexpr int DM = MODE == kTma ? kVec : MODE;  // direct loads

  // chunk k (full 2048-column chunks only) is group k * NW + warp of every warp
  const int nchunks = wide ? 0 : nck;  // chunks of the standard layout
  // a ring wait that gave up: this warp leaves the streaming loop, and the abort flag makes
  // every other warp's next wait give up at once
  auto give_up = [&]() {
    werr = true;
    if (lane == 0) *reinterpret_cast<volatile int*>(&st.abort) = 1;
  };
  if (MODE == kTma && rc.fast && !greedy && nchunks > 0 && !(INDIRECT && rc.nd.proc)) {
    // Bootstrap the cut before anything is pushed: the lane maxima of the first chunk, over
    // columns whose counts are zero and that hold no drafted token (their value needs no
    // penalty), bound 128 distinct keys.
    {
      const long long tw = pc.now();
      if (werr || !ring_wait(&st.bars[0], 0u, &st.abort)) give_up();
      pc.add(PW_WAIT, tw);
      pc.stamp(PS_FIRST, tid == 0);
    }
    const uint4 xq = *reinterpret_cast<const uint4*>(smem_ring + warp * (GROUP * 2) + lane * 16);
    uint32_t y[4] = {xq.x, xq.y, xq.z, xq.w};
    if (brow) {
      const uint4 bq = *reinterpret_cast<const uint4*>(smem_ring + sg_b + warp * (GROUP * 2) + lane * 16);
      y[0] = bf2_add(y[0], bq.x);
      y[1] = bf2_add(y[1], bq.y);
      y[2] = bf2_add(y[2], bq.z);
      y[3] = bf2_add(y[3], bq.w);
    }
    uint32_t ok = grow ? smem_ring[sg_g + warp * (GROUP / 8) + lane] : 0xffu;
    if (drow) {
      const int32_t* dp = reinterpret_cast<const int32_t*>(smem_ring + sg_d + warp * (GROUP * 4)) + 8 * lane;
      const int32_t* cp = reinterpret_cast<const int32_t*>(smem_ring + sg_c + warp * (GROUP * 4)) + 8 * lane;
#pragma unroll
      for (int j = 0; j < VPT; ++j)
        if ((dp[j] | (crow ? cp[j] : 0)) != 0) ok &= ~(1u << j);
    }
    for (int t = 0; t < ntok; ++t) {
      const int64_t dl = (int64_t)st.toks[t] - (gcol(warp) + shard);
      if (dl >= 0 && dl < VPT) ok &= ~(1u << dl);
    }
    const uint32_t base = 0xffffu - wloc(gcol(warp));
    uint32_t lm = 0;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const uint32_t h = half_of(y, j);
      if (((ok >> j) & 1u) && (h & 0x7fffu) <= 0x7f80u) lm = umax(lm, (enc16(h) << 16) | (base - (uint32_t)j));
    }
    lane_max_publish(lm, st.vlm, warp, lane, final_of, mm);
    __syncthreads();
    const float t = lane_max_min(st.vlm, lane);
    if (t > w.thr) wtk_raise(w, &st.cut, t, vmin_pair(t, rc), lane);
  }
  int stage = 0;
  uint32_t phase = 0;
  // wide chunks (greedy rows): groups wg * (NW * k + warp) and the next wg - 1
  for (int k = 0; k < (wide && !werr ? nck : 0); ++k) {
    if (!ring_wait(&st.bars[stage], phase, &st.abort)) {
      give_up();
      break;
    }
    const unsigned char* sp = smem_ring + stage * stage_bytes + warp * (GROUP * 2 * wg) + lane * 16;
    const int g0 = wg * (NW * k + warp);
#pragma unroll 1
    for (int h = 0; h < wg; ++h) {
      Raw8 raw;
      const uint4 xq = *reinterpret_cast<const uint4*>(sp + h * (GROUP * 2));
      raw.x[0] = xq.x; raw.x[1] = xq.y; raw.x[2] = xq.z; raw.x[3] = xq.w;
      greedy_group(raw, gcol(g0 + h), VPT);
    }
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&st.rel[stage], 1) == NW - 1) {
        atomicExch(&st.rel[stage], 0);
        if (k + nst < nck) {
          __threadfence_block();
          fence_proxy_async();
          issue_chunk(k + nst, stage);
        }
      }
    }
    if (++stage == nst) {
      stage = 0;
      phase ^= 1u;
    }
  }
  // the remaining groups: standard ring chunks, then direct loads
  for (int k = 0, g = (wide ? wg * NW * nck : 0) + warp; g < ngroups && !werr; ++k, g += NW) {
    const int64_t c = gcol(g);
    const bool staged = k < nchunks;
    const int nv = staged ? VPT : gvalid(g);  // ring groups are whole
    Raw8 raw;
    if (staged) {
      const long long tw = pc.now();
      if (!ring_wait(&st.bars[stage], phase, &st.abort)) {
        give_up();
        break;
      }
      pc.add(PW_WAIT, tw);
      const long long tl = pc.now();
      const unsigned char* sp = smem_ring + stage * stage_bytes;
      const uint4 xq = *reinterpret_cast<const uint4*>(sp + warp * (GROUP * 2) + lane * 16);
      raw.x[0] = xq.x; raw.x[1] = xq.y; raw.x[2] = xq.z; raw.x[3] = xq.w;
#pragma unroll
      for (int j = 0; j < VPT; ++j) raw.d[j] = raw.c[j] = 0;
#pragma unroll
      for (int p = 0; p < 4; ++p) raw.b[p] = 0;
      raw.g = 0xffu;
      if (INDIRECT && rc.nd.proc) {
        // aux values of the group's target ids, gathered as the direct path does
        int64_t col[VPT];
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          col[j] = c + j + a.shard_offset;
          if (j < nv) col[j] = load_index(a.d2t, a.d2t_dtype, col[j]);
        }
        load_aux8<kScalar>(a.params, rc, slot, col, nv, raw);
        if (rc.nd.g) raw.g = load_g8<kScalar>(a.params, gslot, col, nv);
        add_drafted(raw, col, nv, st.toks, ntok);
      }
      if (rdrow) {
        const unsigned char* dp = sp + sg_d + warp * (GROUP * 4) + lane * 32;
        const uint4 u = *reinterpret_cast<const uint4*>(dp);
        const uint4 v = *reinterpret_cast<const uint4*>(dp + 16);
        raw.d[0] = u.x; raw.d[1] = u.y; raw.d[2] = u.z; raw.d[3] = u.w;
        raw.d[4] = v.x; raw.d[5] = v.y; raw.d[6] = v.z; raw.d[7] = v.w;
      }
      if (rcrow) {
        const unsigned char* cp = sp + sg_c + warp * (GROUP * 4) + lane * 32;
        const uint4 u = *reinterpret_cast<const uint4*>(cp);
        const uint4 v = *reinterpret_cast<const uint4*>(cp + 16);
        raw.c[0] = u.x; raw.c[1] = u.y; raw.c[2] = u.z; raw.c[3] = u.w;
        raw.c[4] = v.x; raw.c[5] = v.y; raw.c[6] = v.z; raw.c[7] = v.w;
      }
      if (rbrow) {
        const uint4 u = *reinterpret_cast<const uint4*>(sp + sg_b + warp * (GROUP * 2) + lane * 16);
        raw.b[0] = u.x; raw.b[1] = u.y; raw.b[2] = u.z; raw.b[3] = u.w;
      }
      if (rgrow) raw.g = sp[sg_g + warp * (GROUP / 8) + lane];
      pc.add(PW_LOADS, tl);
    } else {
      load_group<DM, INDIRECT>(a, rc, slot, gslot, xrow, c, nv, raw, st.toks, ntok);
    }
    process_group(raw, c, nv, k);
    if (staged) {
      // this warp has consumed its slice of the stage; the last of the NW warps refills it
      const long long tr = pc.now();
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&st.rel[stage], 1) == NW - 1) {
          atomicExch(&st.rel[stage], 0);
          if (k + nst < nchunks) {
            __threadfence_block();
            fence_proxy_async();
            issue_chunk(k + nst, stage);
          }
        }
      }
      pc.add(PW_RELEASE, tr);
      if (++stage == nst) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  pdl_trigger();
  pc.stamp(PS_WARP0_END, tid == 0);

  // Bounded-wait error path: a CTA whose ring wait gave up writes nothing for its split. It
  // records the error, lets its issued copies land, and marks its unit's ticket failed, so
  // that the row (or multistep request) leaves its outputs unwritten.
  auto fail_split = [&]() {
    if (tid == 0) {
      atomicOr(ws.error, (uint32_t)SONIC_DEVICE_ERR_WAIT);
      ring_drain(st.bars, st.nissued, nst);
    }
    if (MS) {
      if (tid == 0) atomicOr(ws.tickets + req, 1u);
      return;
    }
    arrive_last(ws.tickets + r, splits, &st.flag, true);
  };

  uint64_t* lists = ws.cand + (uint64_t)r * splits * kMaxK;
  if (greedy) {
    pc.flush(warp, lane);
    best = warp_max_u64(best);
    if (lane == 0) atomicMax(&st.best, (unsigned long long)best);
    if (__syncthreads_or(werr)) {
      fail_split();
      return;
    }
    if (tid == 0) {
      stcg64(lists + (int64_t)split * kMaxK, st.best);
      __threadfence();
    }
  } else {
    // (after a failed wait the absorb only reorders shared memory; the CTA then leaves)
    if (w.qn) wtk_absorb(w, q, lane, tq, rc.temp_fast, rc.temp, rc.rtemp);
    if (lane == 0) st.qn[warp] = 0;
    pc.flush(warp, lane);
    if (__syncthreads_or(werr)) {
      fail_split();
      return;
    }
    // the split's top-128 as 64-bit keys with global columns (in warp 0). WIDE: every warp's
    // list is converted first, laid out [NW][128] over the queues (free now), then folded
    // across the warps; else the 32-bit lists are folded and converted
    auto fold_warps = [&](uint64_t (&out)[4]) {
      if constexpr (WIDE) {
        uint64_t (*lists64)[kMaxK] = reinterpret_cast<uint64_t (*)[kMaxK]>(&st.queue[0][0]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t key = st.lists[warp][4 * lane + i];
          uint64_t gk = 0;
          if (key) {
            const uint32_t loc = 0xffffu - (key & 0xffffu);
            const int64_t col = c0 + ((int64_t)(loc >> 8) << 11) + (int64_t)warp * GROUP + (loc & (GROUP - 1));
            gk = ((uint64_t)(key >> 16) << 32) | (uint64_t)(0xffffffffu - (uint32_t)col);
          }
          lists64[warp][4 * lane + i] = gk;
        }
        block_fold<uint64_t>(lists64, warp, lane, out);
      } else {
        uint32_t f[4];
        block_fold(st.lists, warp, lane, f);
#pragma unroll
        for (int j = 0; j < 4; ++j) out[j] = to_global<uint32_t>(f[j], c0);
      }
    };
    uint64_t fin[4];
    fold_warps(fin);
    pc.stamp(PS_FOLD, tid == 0);
    if (warp == 0) {
      // the split holds at least kk finite candidates when list position kk - 1 is taken
      const int jj = (kk - 1) & 3;
      const uint64_t f = jj == 0 ? fin[0] : (jj == 1 ? fin[1] : (jj == 2 ? fin[2] : fin[3]));
      const uint64_t last = __shfl_sync(kFull, f, (kk - 1) >> 2);
      if (lane == 0) st.flag = last != 0;
    }
    __syncthreads();
    if (!st.flag) {
      // fewer than kk finite candidates in this split: redo it keeping -inf logits,
      // through the exact path
      if (tid == 0) row_smem_init(st, pack_cut(__int_as_float(0xff800000), 0u));
      __syncthreads();
      wtk_init(w, st.lists[warp], __int_as_float(0xff800000), lane);
      tq = false;  // the exact path pushes final keys
      for (int gg = warp; gg < ngroups; gg += NW) {
        Raw8 raw;
        load_group<DM, INDIRECT>(a, rc, slot, gslot, xrow, gcol(gg), gvalid(gg), raw, st.toks, ntok);
        wtk_adopt(w, &st.cut, lane);
        exact_group(raw, gcol(gg), gvalid(gg));
        absorb_if_full();
      }
      if (w.qn) wtk_absorb(w, q, lane);
      if (lane == 0) st.qn[warp] = 0;
      __syncthreads();
      fold_warps(fin);
    }
    if (warp == 0) {
      uint64_t* out = lists + (int64_t)split * kMaxK;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint64_t key = fin[j];
        stcg64(out + 4 * lane + j, key);
        // warm L2 with the noise the merge will gather for this candidate (multistep rows
        // draw their noise in ms_verify_kernel: their launch carries no noise pointer)
        if (key && !MS && !cand_out && !(a.flags & SONIC_FLAG_PHILOX) && !a.d2t &&
            (a.target_vocab <= 0 || key_column(key) < a.target_vocab))
          asm volatile("prefetch.global.L2 [%0];" ::"l"(a.gumbel + slot * a.gumbel_stride + key_column(key)));
      }
      __threadfence();
      pc.stamp(PS_LIST, lane == 0);
    }
  }

  if (MS) return;  // multistep rows: ms_verify_kernel merges the lists after this grid
  bool row_failed = false;
  const bool last_cta = arrive_last(ws.tickets + r, splits, &st.flag, false, &row_failed);
  pc.stamp(PS_TICKET, tid == 0);
  if (!last_cta || row_failed) return;  // a failed split: the row's outputs stay unwritten

  // ---- merge + selection ----
  const uint32_t flags = a.flags;
  if (greedy) {
    if (warp != 0) return;
    uint64_t b = 0;
    for (int s = lane; s < splits; s += 32) b = umax(b, ldcg64(lists + (int64_t)s * kMaxK));
    b = warp_max_u64(b);
    int64_t token = greedy_col(b, log2bn);
    // a column outside the row can only come from a workspace that was not zero-filled
    if (token < 0 || token >= a.vocab_size) token = -1;
    else if (a.d2t) token = load_index(a.d2t, a.d2t_dtype, token);
    if (lane == 0) {
      if ((flags & SONIC_FLAG_UPDATE_COUNTS) && token >= 0 && token < P.counts_stride) {
        int32_t* d = P.decode_counts + slot * P.counts_stride + token;
        if (flags & SONIC_FLAG_PREFILL) *d = 1;
        else atomicAdd(d, 1);
      }
      a.tokens[r * a.tokens_stride] = (int32_t)token;
    }
    return;
  }

  uint64_t k[4];
  block_merge_lists(lists, splits, reinterpret_cast<uint64_t*>(&st.queue[0][0]), warp, lane, k);
  pc.stamp(PS_MERGE, tid == 0);
  if (warp != 0) return;
  if (cand_out) {
    // vocab-sharded step 1: the row's 128 best candidates of this shard, global columns
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint64_t key = k[j];
      if (key) key = (key & 0xffffffff00000000ull) | (uint64_t)(0xffffffffu - (uint32_t)(key_column(key) + shard));
      stcg64(cand_out + r * kMaxK + 4 * lane + j, key);
    }
    return;
  }
  select_row(a, r, slot, ind, st.mp, k, lane);
  pc.stamp(PS_SELECT, lane == 0);
}

// ---------------------------------------------------------------------------------------
// plain singular rows: no grammar, counts, bias, d2t or drafted tokens anywhere in the call
// (logits, optional temperature, then the usual masking and selection). Same machinery as
// singular_kernel with wider groups: 16 columns a lane, 512 a warp, 4096-column chunks of
// logits only (8 KB a stage; 3 stages and 4 CTAs an SM for grids of several waves, else 9 stages
// and 3 CTAs).
// ---------------------------------------------------------------------------------------

constexpr int PVPT = 16;               // columns per lane
constexpr int PGROUP = PVPT * 32;      // columns per warp group
constexpr int PCH = PGROUP * NW;       // columns per chunk
constexpr int PSTAGE = PCH * 2;        // bytes per stage
constexpr int PNST_WAVES = 3;         // ring stages of a multi-wave grid: 24 KB, 4 CTAs an SM
constexpr int PNST_ONE = 9;           // of a one-wave grid: 72 KB, more bytes in flight a CTA
constexpr int PQCAP = kMaxK + PGROUP;  // a warp appends at most 512 keys per group
constexpr int PLAIN_MAX_COLS = 128 * NW * PGROUP;  // a CTA's columns: 128 groups a warp (16-bit key index)
constexpr int PLAIN_SLOTS = 148 * 4;                // CTA slots of the multi-wave logits-only kernel (4 an SM)

// 16 logits of one lane, pre-temperature bf16 pairs; `nvalid` columns valid (-inf beyond)
template <int MODE>
__device__ __forceinline__ void load_x16(const uint16_t* xrow, int64_t c, int nvalid, uint32_t (&x)[8]) {
  uint32_t lo[4], hi[4];
  load_x8<MODE>(xrow, c, min(nvalid, 8), lo);
  load_x8<MODE>(xrow, c + 8, max(nvalid - 8, 0), hi);
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    x[p] = lo[p];
    x[4 + p] = hi[p];
  }
}

// half j of x (a runtime j: explicit selects keep x in registers)
__device__ __forceinline__ uint32_t half16(const uint32_t (&x)[8], int j) {
  const int i = j >> 1;
  const uint32_t a = i & 1 ? x[1] : x[0], b = i & 1 ? x[3] : x[2], c = i & 1 ? x[5] : x[4], d = i & 1 ? x[7] : x[6];
  const uint32_t e = i & 2 ? b : a, f = i & 2 ? d : c;
  const uint32_t w = i & 4 ? f : e;
  return (j & 1) ? (w >> 16) : (w & 0xffffu);
}

// MINB: CTAs an SM the registers are budgeted for (4 for grids of several waves, whose CTAs'
// fixed costs then overlap more; 3 for one-wave grids, which take a deeper ring instead).
// MS: the rows of a multistep call (row r is a step of a request, as in singular_kernel's MS
// mode): every CTA writes its list (greedy rows: its best key) to the workspace for
// ms_verify_kernel, with no ticket, merge or selection here.
template <int MODE, int MINB, bool MS>
__global__ void __launch_bounds__(NT, MINB) plain_kernel(const SonicSingularArgs a, int splits, int cols, int log2bn,
                                                      Workspace ws, int nst, uint64_t* cand_out, const MsRows ms) {
  __shared__ __align__(16) RowSmem<uint32_t, PQCAP> st;
  extern __shared__ __align__(128) unsigned char smem_ring[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int64_t r = blockIdx.y;
  const SonicSamplingParams& P = a.params;
  const int64_t c0 = (int64_t)split * cols;
  const int64_t c1 = min((int64_t)a.vocab_size, c0 + cols);
  PhaseClock pc;
  pc.stamp(PS_ENTRY, tid == 0);

  pdl_wait();
  pc.stamp(PS_PDL, tid == 0);

  // The ring's addresses depend on the row alone: its first stages go out before the row's
  // parameters are loaded, so the copies overlap that chain of dependent loads.
  const uint16_t* xrow = (const uint16_t*)a.logits + r * a.logits_stride;
  const int nchunks = MODE == kTma ? (int)((c1 - c0) / PCH) : 0;
  auto issue_chunk = [&](int i, int stage) {  // one thread
    uint64_t* bar = &st.bars[stage];
    ++st.nissued[stage];
    mbar_expect_tx(bar, (uint32_t)PSTAGE);
    bulk_load(smem_ring + stage * PSTAGE, xrow + c0 + (int64_t)i * PCH, PSTAGE, bar);
  };
  if (MODE == kTma && tid == 0) {
    for (int i = 0; i < nst; ++i) {
      mbar_init(&st.bars[i], 1);
      st.rel[i] = 0;
      st.nissued[i] = 0;
    }
    mbar_init(&st.stall_bar, 1);
    mbar_fence_init();
    for (int i = 0; i < min(nchunks, nst); ++i) issue_chunk(i, i);
  }

  auto drain = [&]() {  // leaving early: the copies already issued land before the CTA leaves
    if (MODE == kTma && tid == 0)
      for (int i = 0; i < min(nchunks, nst); ++i) mbar_wait_bounded(&st.bars[i], 0u, WAIT_LIMIT);
  };
  // MS: row r is step `step` of multistep request `req`
  int64_t req = r, margin = 0;
  int step = 0;
  if (MS && !ms_row(ms, r, req, step, margin)) {
    drain();
    return;
  }
  const int64_t slot = load_slot(P, req);
  if (slot < 0 || (P.num_slots > 0 && slot >= P.num_slots)) {
    if (!MS && split == 0 && tid == 0) a.tokens[r * a.tokens_stride] = -1;
    drain();
    return;
  }
  const SlotScalars sc = load_slot_scalars(P, slot);
  const uint32_t ind = sc.ind;
  const RowConsts rc = row_consts(P, sc);
  // vocab-sharded step 1 (cand_out) keeps greedy rows' candidates too: exact path, top-128
  const bool greedy = (ind & 0x40) != 0 && !cand_out;
  const int kk = needed_candidates(a, sc, MS);  // exact leading candidates needed
  const int mm = (kk + NW - 1) / NW;               // of them per warp (cut rules)
  if (tid == 0) {
    st.abort = 0;
    st.best = 0ull;
    st.mp = mask_params(P, sc);
    row_smem_init(st, pack_cut(kFiniteFloor, rc.fast ? vmin_pair(kFiniteFloor, rc) : 0u));
  }
  __syncthreads();
  bool werr = false;
  if ((a.flags & SONIC_FLAG_DEBUG_STALL_RING) && MODE == kTma && nchunks > 0) {
    // diagnostics: a wait that runs out, then the same error path as a real timeout
    if (!mbar_wait_bounded(&st.stall_bar, 0u, STALL_TEST_LIMIT)) werr = true;
    if (werr && lane == 0) *reinterpret_cast<volatile int*>(&st.abort) = 1;
  }
  auto give_up = [&]() {
    werr = true;
    if (lane == 0) *reinterpret_cast<volatile int*>(&st.abort) = 1;
  };

  uint32_t* q = st.queue[warp];
  WarpTopK<uint32_t> w;
  wtk_init(w, st.lists[warp], kFiniteFloor, lane);
  uint64_t best = 0;
  bool tq = rc.fast && rc.nd.temp;  // fast-path queues hold pre-temperature keys
  auto final_of = [&](float v) { return final_value(v, rc); };
  // Greedy rows: bf16(x / t) is monotone in the logit x for a temperature t in (0, max], so a
  // column whose logit is below the warp's floor (the smallest bf16 logit whose final value
  // reaches the warp's best key) has a strictly smaller key. A lane keys its 16 columns
  // exactly only when one of them is not below the floor (NaN logits always are keyed).
  const bool gfl = greedy && (!rc.nd.temp || (rc.temp > 0.0f && rc.temp <= 3.3895313892515355e+38f));
  uint32_t gf2 = 0xff80ff80u;  // the floor as a bf16 pair (-inf: every column)
  uint64_t gbest = 0;          // the warp's best key when the floor was set

  auto absorb_if_full = [&]() {
    if (w.qn >= kMaxK) {
      const long long ta = pc.now();
      const float t = absorbed_cut(w, wtk_absorb(w, q, lane, tq, rc.temp_fast, rc.temp, rc.rtemp, kk), st.v16, warp,
                                   lane, mm);
      if (t > w.thr) wtk_raise(w, &st.cut, t, rc.fast ? vmin_pair(t, rc) : 0u, lane);
      pc.add(PW_ABSORB, ta);
      pc.count(PW_ABSORBS, 1);
    }
  };
  // queue the keys of the set bits of m (16 columns starting at c)
  // Warp-local key index: the warp's k-th group (columns c0 + (8k + warp) * 512 + [0, 512))
  // has local columns k * 512 + [0, 512). It grows with the column inside the warp's share and
  // fits 16 bits for up to 128 groups a warp (PLAIN_MAX_COLS columns a CTA). Lists of
  // different warps are merged only as 64-bit keys with global columns (warp_global).
  auto warp_local = [&](int64_t c) { return (uint32_t)((((c - c0) >> 12) << 9) | ((c - c0) & (PGROUP - 1))); };
  auto push16 = [&](const uint32_t (&y)[8], uint32_t m, int64_t c, bool tempered) {
    const long long tpp = pc.now();
    pc.count(PW_PUSHED, (unsigned long long)__popc(m));
    int excl;
    const int total = warp_offsets(__popc(m), lane, excl);
    int pos = w.qn + excl;
    const uint32_t base = 0xffffu - warp_local(c);
    while (m) {
      const int j = __ffs(m) - 1;
      m &= m - 1;
      uint32_t h = half16(y, j);
      if (tempered) h = f2bf(final_value(bf2f((uint16_t)h), rc));
      q[pos++] = (enc16(h) << 16) | (base - (uint32_t)j);
    }
    w.qn += total;
    pc.add(PW_PUSHPATH, tpp);
  };
  int adopt_tick = 0;
  auto process16 = [&](const uint32_t (&x)[8], int64_t c, int nvalid, bool exact) {
    const long long tp = pc.now();
    pc.count(PW_GROUPS, 1);
    const uint32_t valid = nvalid >= PVPT ? 0xffffu : ((1u << max(nvalid, 0)) - 1u);
    if (greedy) {
      bool pass = true;
      if (gfl) {
        uint32_t below = 0xffffffffu;
#pragma unroll
        for (int p = 0; p < 8; ++p)
          below &= __hlt2_mask(*reinterpret_cast<const __nv_bfloat162*>(&x[p]),
                               *reinterpret_cast<const __nv_bfloat162*>(&gf2));
        pass = below != 0xffffffffu;
      }
      bool rose = false;
      if (pass) {
        pc.count(PW_PUSHED, 1);  // diagnostics: lanes that key their columns
#pragma unroll
        for (int j = 0; j < PVPT; ++j) {
          if ((valid >> j) & 1u) {
            const uint32_t h =
                rc.nd.temp ? (uint32_t)f2bf(final_value(bf2f((uint16_t)half16(x, j)), rc)) : half16(x, j);
            const uint64_t k = greedy_key_bits(h, c + j, log2bn);
            rose |= k > best;
            best = umax(best, k);
          }
        }
      }
      // raise the warp's floor when its best key rose (a NaN or -inf best leaves it)
      if (gfl && __any_sync(kFull, rose)) {
        const uint64_t wb = warp_max_u64(best);
        if (wb > gbest) {
          gbest = wb;
          const uint32_t hb = dec16((uint32_t)(wb >> 48));
          const float tv = bf2f((uint16_t)hb);
          if (tv > __int_as_float(0xff800000)) {
            const uint32_t f = rc.nd.temp ? (uint32_t)f2bf(greedy_floor(tv, rc.temp_fast, rc.temp, rc.rtemp)) : hb;
            gf2 = f | (f << 16);
          }
        }
      }
      pc.add(PW_PROCESS, tp);
      return;
    }
    // the CTA cut of the other warps, adopted every other group (a stale cut only admits more)
    if (exact || (++adopt_tick & 1)) wtk_adopt(w, &st.cut, lane);
    uint32_t m = 0;
    if (rc.fast && !exact) {
      const uint32_t lo[4] = {x[0], x[1], x[2], x[3]}, hi[4] = {x[4], x[5], x[6], x[7]};
      m = (ge_mask8(lo, w.vmin2) | (ge_mask8(hi, w.vmin2) << 8)) & valid;
      if (__any_sync(kFull, m)) push16(x, m, c, false);
    } else {
      const float thr = w.thr;
#pragma unroll
      for (int j = 0; j < PVPT; ++j)
        if (((valid >> j) & 1u) && final_value(bf2f((uint16_t)half16(x, j)), rc) >= thr) m |= 1u << j;
      if (__any_sync(kFull, m)) push16(x, m, c, rc.nd.temp);
    }
    absorb_if_full();
    pc.add(PW_PROCESS, tp);
  };

  // groups of this warp: g = warp, warp + NW, ...; columns [c0 + g * PGROUP, +PGROUP)
  const int ngroups = (int)((c1 - c0 + PGROUP - 1) / PGROUP);
  auto gcol = [&](int g) { return c0 + (int64_t)g * PGROUP + (int64_t)PVPT * lane; };
  auto gvalid = [&](int g) { return (int)max((int64_t)0, min((int64_t)PVPT, c1 - gcol(g))); };
  constexpr int DM = MODE == kTma ? kVec : MODE;
  if (MODE == kTma && rc.fast && !greedy && nchunks > 0) {
    // cut bootstrap from the first chunk's lane maxima (see lane_max_publish)
    if (werr || !ring_wait(&st.bars[0], 0u, &st.abort)) give_up();
    const unsigned char* sp = smem_ring + warp * (PGROUP * 2) + lane * 32;
    const uint4 u0 = *reinterpret_cast<const uint4*>(sp), u1 = *reinterpret_cast<const uint4*>(sp + 16);
    const uint32_t x[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    const uint32_t base = (uint32_t)(0xffff - (int)(gcol(warp) - c0));
    uint32_t lm = 0;
#pragma unroll
    for (int j = 0; j < PVPT; ++j) {
      const uint32_t h = half16(x, j);
      if ((h & 0x7fffu) <= 0x7f80u) lm = umax(lm, (enc16(h) << 16) | (base - (uint32_t)j));
    }
    lane_max_publish(lm, st.vlm, warp, lane, final_of, mm);
    __syncthreads();
    const float t = lane_max_min(st.vlm, lane);
    if (t > w.thr) wtk_raise(w, &st.cut, t, vmin_pair(t, rc), lane);
  }

  // Cut refresh: each lane keeps the running maximum of the logits it has streamed through
  // the ring (bf16 pairs). As for the bootstrap, the m-th largest lane maximum of every warp
  // bounds 8m distinct columns, so the smallest over the warps is a valid cut; a stale value
  // of another warp is smaller, so also valid. Refreshed after the warp's groups 1, 3 and 7:
  // early, when the cut is still low and most groups push.
  const bool refresh = MODE == kTma && rc.fast && !greedy && nchunks > 0;
  uint32_t lmv = 0xff80ff80u;
  int stage = 0;
  uint32_t phase = 0;
  int64_t cg = gcol(warp);  // the lane's first column of group g, advanced with g
  for (int k = 0, g = warp; g < ngroups && !werr; ++k, g += NW, cg += (int64_t)NW * PGROUP) {
    const int64_t c = cg;
    const bool staged = k < nchunks;
    uint32_t x[8];
    const int nv = staged ? PVPT : gvalid(g);  // ring groups are whole
    if (staged) {
      const long long tw = pc.now();
      if (!ring_wait(&st.bars[stage], phase, &st.abort)) {
        give_up();
        break;
      }
      pc.add(PW_WAIT, tw);
      if (k == 0) pc.stamp(PS_FIRST, tid == 0);
      const unsigned char* sp = smem_ring + stage * PSTAGE + warp * (PGROUP * 2) + lane * 32;
      const uint4 u0 = *reinterpret_cast<const uint4*>(sp), u1 = *reinterpret_cast<const uint4*>(sp + 16);
      x[0] = u0.x; x[1] = u0.y; x[2] = u0.z; x[3] = u0.w;
      x[4] = u1.x; x[5] = u1.y; x[6] = u1.z; x[7] = u1.w;
    } else {
      load_x16<DM>(xrow, c, nv, x);
    }
    process16(x, c, nv, false);
    if (refresh && staged) {
      const uint32_t m01 = bf2_max(bf2_max(x[0], x[1]), bf2_max(x[2], x[3]));
      const uint32_t m23 = bf2_max(bf2_max(x[4], x[5]), bf2_max(x[6], x[7]));
      lmv = bf2_max(lmv, bf2_max(m01, m23));
      if (k <= 63 && k > 0 && (k & (k + 1)) == 0) {  // k = 1, 3, 7, 15, 31, 63
        const uint32_t lo = lmv & 0xffffu, hi = lmv >> 16;
        const uint32_t h = enc16(lo) >= enc16(hi) ? lo : hi;
        lane_max_publish((h & 0x7fffu) <= 0x7f80u ? enc16(h) << 16 : 0u, st.vlm, warp, lane, final_of, mm);
        __syncwarp();
        const float t = lane_max_min(st.vlm, lane);
        if (t > w.thr) wtk_raise(w, &st.cut, t, vmin_pair(t, rc), lane);
      }
    }
    if (staged) {
      // this warp has consumed its slice of the stage; the last of the NW warps refills it
      const long long tr = pc.now();
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&st.rel[stage], 1) == NW - 1) {
          atomicExch(&st.rel[stage], 0);
          if (k + nst < nchunks) {
            __threadfence_block();
            fence_proxy_async();
            issue_chunk(k + nst, stage);
          }
        }
      }
      pc.add(PW_RELEASE, tr);
      if (++stage == nst) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  pdl_trigger();
  pc.stamp(PS_WARP0_END, tid == 0);

  // bounded-wait error path (see singular_kernel): no outputs for this row (multistep: for
  // its request, which ms_verify_kernel sees marked)
  auto fail_split = [&]() {
    if (tid == 0) {
      atomicOr(ws.error, (uint32_t)SONIC_DEVICE_ERR_WAIT);
      if (MODE == kTma) ring_drain(st.bars, st.nissued, nst);
      if (MS) atomicOr(ws.tickets + req, 1u);
    }
    if (!MS) arrive_last(ws.tickets + r, splits, &st.flag, true);
  };

  uint64_t* lists = ws.cand + (uint64_t)r * splits * kMaxK;
  // one CTA covers the whole row: no workspace list, no ticket, no merge across CTAs
  const bool whole_row = !MS && splits == 1;
  if (greedy) {
    pc.flush(warp, lane);
    best = warp_max_u64(best);
    if (lane == 0) atomicMax(&st.best, (unsigned long long)best);
    if (__syncthreads_or(werr)) {
      fail_split();
      return;
    }
    if (tid == 0 && !whole_row) {
      stcg64(lists + (int64_t)split * kMaxK, st.best);
      __threadfence();
    }
  } else {
    // (after a failed wait the absorb only reorders shared memory; the CTA then leaves)
    if (w.qn) wtk_absorb(w, q, lane, tq, rc.temp_fast, rc.temp, rc.rtemp);
    pc.flush(warp, lane);
    if (__syncthreads_or(werr)) {
      fail_split();
      return;
    }
    // every warp's list as 64-bit keys with global columns, laid out [NW][128] over the
    // queues (free now), then one fold across the warps
    uint64_t (*lists64)[kMaxK] = reinterpret_cast<uint64_t (*)[kMaxK]>(&st.queue[0][0]);
    auto fold_warps = [&](uint64_t (&fin)[4]) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t key = st.lists[warp][4 * lane + i];
        uint64_t gk = 0;
        if (key) {
          const uint32_t loc = 0xffffu - (key & 0xffffu);
          const int64_t col = c0 + ((int64_t)(loc >> 9) << 12) + (int64_t)warp * PGROUP + (loc & (PGROUP - 1));
          gk = ((uint64_t)(key >> 16) << 32) | (uint64_t)(0xffffffffu - (uint32_t)col);
        }
        lists64[warp][4 * lane + i] = gk;
      }
      block_fold<uint64_t>(lists64, warp, lane, fin);
    };
    uint64_t fin[4];
    fold_warps(fin);
    pc.stamp(PS_FOLD, tid == 0);
    if (warp == 0) {
      // the CTA holds at least kk finite candidates when list position kk - 1 is taken
      const int jj = (kk - 1) & 3;
      const uint64_t f = jj == 0 ? fin[0] : (jj == 1 ? fin[1] : (jj == 2 ? fin[2] : fin[3]));
      const uint64_t last = __shfl_sync(kFull, f, (kk - 1) >> 2);
      if (lane == 0) st.flag = last != 0;
    }
    __syncthreads();
    if (!st.flag) {
      // fewer than kk finite candidates in the CTA's columns: redo them keeping -inf logits
      if (tid == 0) row_smem_init(st, pack_cut(__int_as_float(0xff800000), 0u));
      __syncthreads();
      wtk_init(w, st.lists[warp], __int_as_float(0xff800000), lane);
      tq = false;
      for (int gg = warp; gg < ngroups; gg += NW) {
        uint32_t x[8];
        load_x16<DM>(xrow, gcol(gg), gvalid(gg), x);
        process16(x, gcol(gg), gvalid(gg), true);
      }
      if (w.qn) wtk_absorb(w, q, lane);
      __syncthreads();
      fold_warps(fin);
    }
    if (warp == 0) {
      if (whole_row) {
#pragma unroll
        for (int i = 0; i < 4; ++i) lists64[0][4 * lane + i] = fin[i];
      } else {
        uint64_t* out = lists + (int64_t)split * kMaxK;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint64_t key = fin[j];
          stcg64(out + 4 * lane + j, key);
          if (key && !cand_out && a.gumbel && !(a.flags & SONIC_FLAG_PHILOX) &&
              (a.target_vocab <= 0 || key_column(key) < a.target_vocab))
            asm volatile("prefetch.global.L2 [%0];" ::"l"(a.gumbel + slot * a.gumbel_stride + key_column(key)));
        }
        __threadfence();
      }
    }
  }

  if (MS) return;  // multistep rows: ms_verify_kernel merges the lists after this grid
  if (!whole_row) {
    bool row_failed = false;
    if (!arrive_last(ws.tickets + r, splits, &st.flag, false, &row_failed) || row_failed) return;
  }

  if (greedy) {
    if (warp != 0) return;
    uint64_t b = 0;
    if (whole_row) b = st.best;
    else
      for (int s = lane; s < splits; s += 32) b = umax(b, ldcg64(lists + (int64_t)s * kMaxK));
    b = warp_max_u64(b);
    int64_t token = greedy_col(b, log2bn);
    if (token < 0 || token >= a.vocab_size) token = -1;
    if (lane == 0) a.tokens[r * a.tokens_stride] = (int32_t)token;
    return;
  }
  uint64_t k[4];
  if (whole_row) {
    if (warp != 0) return;
    const uint64_t (*lists64)[kMaxK] = reinterpret_cast<const uint64_t (*)[kMaxK]>(&st.queue[0][0]);
#pragma unroll
    for (int i = 0; i < 4; ++i) k[i] = lists64[0][4 * lane + i];
    pc.stamp(PS_MERGE, lane == 0);
  } else {
    block_merge_lists(lists, splits, reinterpret_cast<uint64_t*>(&st.queue[0][0]), warp, lane, k);
    if (warp != 0) return;
  }
  if (cand_out) {
    // vocab-sharded step 1: the row's 128 best candidates of this shard, global columns
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint64_t key = k[j];
      if (key)
        key = (key & 0xffffffff00000000ull) | (uint64_t)(0xffffffffu - (uint32_t)(key_column(key) + a.shard_offset));
      stcg64(cand_out + r * kMaxK + 4 * lane + j, key);
    }
    return;
  }
  select_row(a, r, slot, ind, st.mp, k, lane);
  pc.stamp(PS_SELECT, lane == 0);
}

// ---------------------------------------------------------------------------------------
// vocab-sharded singular, step 3: merge the ranks' candidate lists of a row (gathered
// [world][rows][128] keys with global columns) and select, identically on every rank
// ---------------------------------------------------------------------------------------

__global__ void __launch_bounds__(NT) merge_candidates_kernel(const SonicSingularArgs a, const uint64_t* gathered,
                                                              int world) {
  __shared__ __align__(16) uint64_t xchg[NW][kMaxK];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = blockIdx.x;
  const SonicSamplingParams& P = a.params;
  pdl_wait();
  const int64_t slot = load_slot(P, r);
  if (slot < 0 || (P.num_slots > 0 && slot >= P.num_slots)) {
    if (threadIdx.x == 0) a.tokens[r * a.tokens_stride] = -1;
    return;
  }
  const uint32_t ind = P.indicators[slot];
  uint64_t k[4];
  block_merge_lists(gathered + r * kMaxK, world, &xchg[0][0], warp, lane, k, (int64_t)a.rows * kMaxK);
  pdl_trigger();
  if (warp != 0) return;
  if (ind & 0x40) {
    // greedy: the best candidate (largest value, lowest global column)
    const uint64_t best = __shfl_sync(kFull, k[0], 0);
    int64_t token = best ? key_column(best) : -1;
    if (token >= a.vocab_size) token = -1;
    if (lane == 0) {
      if ((a.flags & SONIC_FLAG_UPDATE_COUNTS) && token >= 0 && token < P.counts_stride) {
        int32_t* d = P.decode_counts + slot * P.counts_stride + token;
        if (a.flags & SONIC_FLAG_PREFILL) *d = 1;
        else atomicAdd(d, 1);
      }
      a.tokens[r * a.tokens_stride] = (int32_t)token;
    }
    return;
  }
  select_row(a, r, slot, ind, load_mask_params(P, slot), k, lane);
}

// ---------------------------------------------------------------------------------------
// bounded top-k (ops/topk/bitpack.py:99 + ops/topk/unpack.py:312)
// ---------------------------------------------------------------------------------------

template <bool F32, bool VEC>
__device__ __forceinline__ void load_vals8(const unsigned char* xrow, int64_t c, int nvalid, float (&x)[VPT]) {
  if (F32) {
    const float* xr = (const float*)xrow;
    if (VEC && nvalid == VPT) {
      const uint4 p = ld_stream(xr + c), u = ld_stream(xr + c + 4);
      x[0] = __uint_as_float(p.x); x[1] = __uint_as_float(p.y); x[2] = __uint_as_float(p.z);
      x[3] = __uint_as_float(p.w); x[4] = __uint_as_float(u.x); x[5] = __uint_as_float(u.y);
      x[6] = __uint_as_float(u.z); x[7] = __uint_as_float(u.w);
    } else {
#pragma unroll
      for (int j = 0; j < VPT; ++j) x[j] = j < nvalid ? __ldcs(xr + c + j) : 0.0f;
    }
  } else {
    uint32_t wv[4];
    load_x8<VEC ? kVec : kScalar>((const uint16_t*)xrow, c, nvalid, wv);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      x[2 * p] = bf2_lo(wv[p]);
      x[2 * p + 1] = bf2_hi(wv[p]);
    }
  }
}

template <int MODE, bool F32>
__global__ void __launch_bounds__(NT) topk_kernel(const SonicTopKArgs a, int splits, int cols, Workspace ws) {
  using K = typename std::conditional<F32, uint64_t, uint32_t>::type;
  constexpr int EB = F32 ? 4 : 2;  // element bytes
  constexpr bool VEC = MODE == kVec;
  __shared__ __align__(16) RowSmem<K> st;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int64_t r = blockIdx.y;
  const int64_t c0 = (int64_t)split * cols;
  const int64_t c1 = min((int64_t)a.vocab_size, c0 + cols);
  const unsigned char* xrow = (const unsigned char*)a.logits + r * a.logits_stride * EB;

  pdl_wait();
  if (tid == 0) row_smem_init(st, pack_cut(kFiniteFloor, 0u));
  __syncthreads();

  K* q = st.queue[warp];
  WarpTopK<K> w;
  wtk_init(w, st.lists[warp], kFiniteFloor, lane);
  const int kk = min(max(a.k, 1), kMaxK);  // only the first k keys of each split are exact
  const int mm = (kk + NW - 1) / NW;

  auto consume = [&](const float (&x)[VPT], int64_t c, int nvalid) {
    wtk_adopt(w, &st.cut, lane);
    const float thr = w.thr;
    unsigned m = 0;
#pragma unroll
    for (int j = 0; j < VPT; ++j)
      if (j < nvalid && x[j] >= thr) m |= 1u << j;
    if (__any_sync(kFull, m)) {
      K key[VPT];
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int local = (int)(c + j - c0);
        if (F32)
          key[j] = (K)(((uint64_t)enc32(x[j]) << 32) | (uint64_t)(0xffffffffu - (uint32_t)local));
        else
          key[j] = (K)((enc16(f2bf(x[j])) << 16) | (uint32_t)(0xffff - local));
      }
      wtk_push(w, q, key, m, lane);
    }
    if (w.qn >= kMaxK) {
      const float t = absorbed_cut(w, wtk_absorb(w, q, lane, false, false, 1.0f, 1.0f, kk), st.v16, warp, lane, mm);
      if (t > w.thr) wtk_raise(w, &st.cut, t, 0u, lane);
    }
  };

  const int ngroups = (int)((c1 - c0 + GROUP - 1) / GROUP);
  auto gcol = [&](int g) { return c0 + (int64_t)g * GROUP + (int64_t)VPT * lane; };
  auto gvalid = [&](int g) { return (int)max((int64_t)0, min((int64_t)VPT, c1 - gcol(g))); };
  auto prefetch_group = [&](int g) {
    if (!VEC || lane != 0 || g >= ngroups) return;
    const int64_t cc = c0 + (int64_t)g * GROUP;
    if (cc + GROUP <= c1) prefetch_l2(xrow + cc * EB, GROUP * EB);
  };
  for (int k = 1; k <= PF_GROUPS; ++k) prefetch_group(warp + k * NW);

  float xa[VPT], xb[VPT];
  if (warp < ngroups) load_vals8<F32, VEC>(xrow, gcol(warp), gvalid(warp), xa);
  for (int g = warp; g < ngroups; g += NW) {
    const bool more = g + NW < ngroups;
    if (more) load_vals8<F32, VEC>(xrow, gcol(g + NW), gvalid(g + NW), xb);
    prefetch_group(g + (PF_GROUPS + 1) * NW);
    consume(xa, gcol(g), gvalid(g));
    if (more) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) xa[j] = xb[j];
    }
  }
  pdl_trigger();

  if (w.qn) wtk_absorb(w, q, lane);
  K fin[4];
  block_fold(st.lists, warp, lane, fin);
  if (warp == 0) {
    // the split holds at least kk finite values when list position kk - 1 is taken
    const int jj = (kk - 1) & 3;
    const K f = jj == 0 ? fin[0] : (jj == 1 ? fin[1] : (jj == 2 ? fin[2] : fin[3]));
    const K last = __shfl_sync(kFull, f, (kk - 1) >> 2);
    if (lane == 0) st.flag = last != 0;
  }
  __syncthreads();
  if (!st.flag) {
    // fewer than kk finite values in this split: redo it keeping -inf
    if (tid == 0) row_smem_init(st, pack_cut(__int_as_float(0xff800000), 0u));
    __syncthreads();
    wtk_init(w, st.lists[warp], __int_as_float(0xff800000), lane);
    for (int gg = warp; gg < ngroups; gg += NW) {
      float x[VPT];
      load_vals8<F32, VEC>(xrow, gcol(gg), gvalid(gg), x);
      consume(x, gcol(gg), gvalid(gg));
    }
    if (w.qn) wtk_absorb(w, q, lane);
    block_fold(st.lists, warp, lane, fin);
  }
  uint64_t* lists = ws.cand + (uint64_t)r * splits * kMaxK;
  if (warp == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) stcg64(lists + (int64_t)split * kMaxK + 4 * lane + j, to_global<K>(fin[j], c0));
    __threadfence();
  }
  if (!arrive_last(ws.tickets + r, splits, &st.flag)) return;

  uint64_t k[4];
  block_merge_lists(lists, splits, reinterpret_cast<uint64_t*>(&st.queue[0][0]), warp, lane, k);
  if (warp != 0) return;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * lane + j;
    if (i >= a.k) continue;
    const uint32_t e = (uint32_t)(k[j] >> 32);
    const int64_t col = key_column(k[j]);
    const int64_t o = r * a.k + i;
    const float val = F32 ? dec32(e) : bf2f((uint16_t)dec16(e));
    if (a.values_dtype == SONIC_DTYPE_F32)
      ((float*)a.values)[o] = val;
    else
      ((uint16_t*)a.values)[o] = F32 ? f2bf(val) : (uint16_t)dec16(e);
    if (a.indices_dtype == SONIC_DTYPE_I64)
      ((int64_t*)a.indices)[o] = col;
    else
      ((int32_t*)a.indices)[o] = (int32_t)col;
  }
}

// ---------------------------------------------------------------------------------------
// fused multistep (ops/prologue.py:272 + ops/multistep.py:76 + ops/verify.py:244): the
// rows of every request stream through singular_kernel in MS mode (per-split top-128
// lists in the workspace); then one CTA per request merges each row's lists, writes the
// stage-2 buffers and runs the chain verification
// ---------------------------------------------------------------------------------------

struct MsSmem {
  int32_t drafted[MS_MAX_STEPS];
  float u[MS_MAX_STEPS];   // acceptance uniform of each step
  float qd[MS_MAX_STEPS];  // draft probability of each drafted token (stochastic drafts)
  float prob[MS_MAX_STEPS][kMaxK];
  int32_t cand[MS_MAX_STEPS][kMaxK];
  float score[MS_MAX_STEPS][kMaxK];  // residual-draw score of each candidate, were the chain to stop at the row
  float lz[MS_MAX_STEPS][kMaxK];     // log-probability of each candidate (top-Z outputs)
  int64_t gsel[MS_MAX_STEPS];
};

__global__ void __launch_bounds__(NT) ms_verify_kernel(const SonicMultistepArgs a, int splits, int log2bn,
                                                       Workspace ws) {
  __shared__ __align__(16) MsSmem sm;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t b = blockIdx.x;
  const SonicSamplingParams& P = a.params;
  const int G = a.lookahead;

  // Everything before pdl_wait reads only the call's inputs (never the rows kernel's candidate
  // lists or failure marks), so under PDL it overlaps the rows kernel's tail. The rows kernel
  // waited for every earlier kernel of the stream before it let this grid start.
  int64_t margin, T;
  if (a.cu_seqlens) {
    margin = a.cu_seqlens[b];
    T = a.cu_seqlens[b + 1] - margin;
  } else {
    margin = b * (G + 1);
    T = G + 1;
  }
  // a request holds 1..gamma+1 rows; anything else is a malformed cu_seqlens
  T = max((int64_t)1, min(T, (int64_t)(G + 1)));
  const int64_t slot = load_slot(P, b);
  if (slot < 0 || (P.num_slots > 0 && slot >= P.num_slots) || margin < 0 || margin + T > a.total_rows) {
    if (tid == 0) a.offsets[b] = -1;
    return;
  }
  const uint32_t ind = P.indicators[slot];
  const bool greedy = (ind & 0x40) != 0;
  const bool stochastic_q = a.draft_probs && !(ind & 0x800) && !greedy;
  // per-slot parameters of the masking and the top-Z outputs, loaded with the other inputs
  const MaskParams mp = load_mask_params(P, slot);
  if (tid < T) {
    const int32_t d = a.drafted_tokens[margin + tid];
    sm.drafted[tid] = d;
    // the acceptance loop's per-step inputs, loaded once and in parallel
    if (!greedy && tid < T - 1) {
      sm.u[tid] = (a.flags & SONIC_FLAG_PHILOX) ? philox_acceptance(a.philox_seed, a.philox_offset + tid, (uint32_t)slot)
                                                : bf2f(a.uniform[slot * a.uniform_stride + tid]);
      float q = 1.0f;
      if (stochastic_q && d >= 0 && d < a.vocab_size) {
        const int64_t qi = slot * a.draft_stride + tid * a.draft_step_stride + d;
        q = a.draft_dtype == SONIC_DTYPE_F32 ? ((const float*)a.draft_probs)[qi]
                                             : bf2f(((const uint16_t*)a.draft_probs)[qi]);
      }
      sm.qd[tid] = q;
    }
  }
  __syncthreads();

  pdl_wait();
  // A CTA of this request's rows gave up a bounded wait (singular_kernel's error path): the
  // request writes no outputs, and its mark is cleared for the next call. The mark is loaded
  // together with the rows' lists and checked before the first output is written.
  const uint32_t failed = ldcg32(ws.tickets + b);

  // ---- per-row merge (warp w handles rows w, w+8, ...) ----
  for (int s = warp; s < T; s += NT / 32) {
    const uint64_t* lists = ws.cand + (margin + s) * splits * kMaxK;
    if (greedy) {
      uint64_t bk = 0;
      for (int q = lane; q < splits; q += 32) bk = umax(bk, ldcg64(lists + (int64_t)q * kMaxK));
      bk = warp_max_u64(bk);
      const int64_t g = greedy_col(bk, log2bn);
      if (lane == 0) {
        sm.gsel[s] = g;
        if (a.indices && !failed) a.indices[margin * kMaxK + s] = (int32_t)g;
      }
    } else {
      uint64_t k[4];
      warp_fold_lists(lists, splits, lane, k);
      float v[4];
      int64_t idx[4];
      decode_keys(k, v, idx);
      // What the residual draw needs of these candidates (their noise and draft probabilities),
      // loaded now for every row: the loads overlap the masking and the softmax below, and the
      // row's scores are ready when the acceptance loop ends.
      uint16_t gcv[4] = {0, 0, 0, 0};
      float qcv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (idx[j] < 0 || idx[j] >= a.vocab_size) continue;
        if (!(a.flags & SONIC_FLAG_PHILOX)) gcv[j] = a.gumbel[slot * a.gumbel_stride + s * a.gumbel_step_stride + idx[j]];
        if (stochastic_q && s < T - 1) {
          const int64_t qi = slot * a.draft_stride + s * a.draft_step_stride + idx[j];
          qcv[j] = a.draft_dtype == SONIC_DTYPE_F32 ? ((const float*)a.draft_probs)[qi]
                                                    : bf2f(((const uint16_t*)a.draft_probs)[qi]);
        }
      }
      const float vmax = __shfl_sync(kFull, v[0], 0);
      float ev[4];
      if (ind & 0x380) warp_masking(mp, ind, v, vmax, lane, ev);
      float ls[4];
      warp_log_softmax(v, vmax, ls);
      const bool want_z = a.max_top_logprobs > 0 && (ind & 0x400) && a.top_logprob_values && P.top_logprobs;
      const int zrow = min(mp.top_logprobs, a.max_top_logprobs);
      const bool stochastic_draft = a.draft_probs && !(ind & 0x800);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = 4 * lane + j;
        const float p = dexp(ls[j]);
        sm.prob[s][i] = p;
        sm.cand[s][i] = (int32_t)idx[j];
        if (want_z && i < zrow) sm.lz[s][i] = dlog(p);
        // rejection_sample (verify.py:157-241) for a chain that stops at this row: the residual
        // max(p - q, 0) of a stochastic draft, p without the drafted token for a greedy draft,
        // p itself past the last draft; then log(residual) - noise. A column outside the row
        // can only come from a workspace that was not zero-filled: it scores -inf.
        const bool bad = idx[j] < 0 || idx[j] >= a.vocab_size;
        float rr;
        if (bad)
          rr = 0.0f;
        else if (s == T - 1)
          rr = p;
        else if (!stochastic_draft)
          rr = (idx[j] == sm.drafted[s]) ? 0.0f : p;
        else {
          rr = __fsub_rn(p, qcv[j]);
          rr = rr < 0.0f ? 0.0f : (rr > 1.0f ? 1.0f : rr);
        }
        const float g = bad ? 0.0f
                            : (a.flags & SONIC_FLAG_PHILOX)
                                  ? philox_log_exponential(a.philox_seed, a.philox_offset + s, (uint32_t)slot,
                                                           (uint32_t)idx[j])
                                  : bf2f(gcv[j]);
        sm.score[s][i] = __fsub_rn(dlog(rr), g);
        if (a.values && !failed) a.values[(margin + s) * kMaxK + i] = p;
        if (a.indices && !failed) a.indices[(margin + s) * kMaxK + i] = (int32_t)idx[j];
      }
    }
  }
  __syncthreads();
  if (failed) {
    if (tid == 0) ws.tickets[b] = 0;
    return;
  }
  if (warp != 0) return;

  // ---- chain verification (verify.py:244-434), one warp ----
  const uint32_t flags = a.flags;
  int32_t dr[MS_MAX_STEPS];
#pragma unroll
  for (int s = 0; s < MS_MAX_STEPS; ++s) dr[s] = (s < T - 1) ? sm.drafted[s] : 0;
  int64_t accepted = 0, token;
  if (greedy) {
    while (accepted < T - 1 && sm.gsel[accepted] == dr[accepted]) ++accepted;
    token = sm.gsel[accepted];
    if ((flags & SONIC_FLAG_UPDATE_COUNTS) && lane == 0)
      for (int64_t s = 0; s <= accepted; ++s)
        if (sm.gsel[s] >= 0 && sm.gsel[s] < P.counts_stride)
          atomicAdd(P.decode_counts + slot * P.counts_stride + sm.gsel[s], 1);
  } else {
    // p(x_s) over the candidates of each row (verify.py:113-127)
    float targets[MS_MAX_STEPS];
#pragma unroll
    for (int s = 0; s < MS_MAX_STEPS; ++s) {
      float t = 0.0f;
      if (s < T) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (sm.cand[s][4 * lane + j] == dr[s]) t = sm.prob[s][4 * lane + j];
#pragma unroll
        for (int d = 16; d >= 1; d >>= 1) t = umax(t, __shfl_xor_sync(kFull, t, d));
      }
      targets[s] = t;
    }
    const bool stochastic_draft = a.draft_probs && !(ind & 0x800);
    for (accepted = 0; accepted < T - 1; ++accepted) {
      float u = sm.u[accepted];
      if (stochastic_draft && dr[accepted] >= 0 && dr[accepted] < a.vocab_size) {
        if (a.draft_dtype == SONIC_DTYPE_F32)
          u = __fmul_rn(u, sm.qd[accepted]);
        else
          u = rbf(__fmul_rn(u, sm.qd[accepted]));
      }
      bool keep = false;
#pragma unroll
      for (int s = 0; s < MS_MAX_STEPS; ++s)
        if (s == accepted) keep = u <= targets[s];
      if (!keep) break;
    }
    // rejection_sample (verify.py:157-241): the accepted row's scores, computed in the merge
    float score[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) score[j] = sm.score[accepted][4 * lane + j];
    const int sel = warp_argmax128(score, lane);
    token = sm.cand[accepted][sel];
    const float psel = sm.prob[accepted][sel];
    if ((flags & SONIC_FLAG_LOGPROBS) && a.logprobs) {
      for (int64_t s = 0; s <= accepted; ++s) {
        float t = 0.0f;
#pragma unroll
        for (int q = 0; q < MS_MAX_STEPS; ++q)
          if (q == s) t = targets[q];
        if (s == accepted) t = psel;
        if (lane == 0) store_float(a.logprobs, a.logprobs_dtype, margin + s, dlog(t));
        if (a.max_top_logprobs > 0 && (ind & 0x400) && a.top_logprob_values && P.top_logprobs) {
          const int z = min(mp.top_logprobs, a.max_top_logprobs);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int i = 4 * lane + j;
            if (i < z) {
              store_float(a.top_logprob_values, a.logprobs_dtype, (margin + s) * a.top_stride + i, sm.lz[s][i]);
              a.top_logprob_tokens[(margin + s) * a.top_stride + i] = sm.cand[s][i];
            }
          }
        }
      }
    }
    if ((flags & SONIC_FLAG_UPDATE_COUNTS) && lane == 0)
      for (int64_t s = 0; s <= accepted; ++s) {
        const int64_t t = s == accepted ? token : (int64_t)sm.drafted[s];
        if (t >= 0 && t < P.counts_stride) atomicAdd(P.decode_counts + slot * P.counts_stride + t, 1);
      }
  }
  if (lane == 0) {
    a.tokens[margin + accepted] = (int32_t)token;
    a.offsets[b] = (int32_t)accepted;
  }
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------

static thread_local std::string g_last_error;

static sonic_status fail(sonic_status code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

static bool aligned(const void* p, size_t a) { return ((uintptr_t)p % a) == 0; }

static int ilog2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

template <typename Kern, typename... Args>
static cudaError_t launch(Kern kern, dim3 grid, size_t smem, cudaStream_t stream, bool pdl, Args... args) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

static sonic_status check_launch(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(SONIC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SONIC_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return SONIC_OK;
}

static sonic_status check_block_n(int32_t block_n) {
  if (block_n < 256 || block_n > 65536 || (block_n & (block_n - 1)))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "block_n must be a power of two in [256, 65536]");
  return SONIC_OK;
}

// 16-byte vector loads of aux rows: every row start and column offset 32-byte aligned
static bool params_vec_ok(const SonicSamplingParams& P, int64_t shard_offset) {
  bool ok = (shard_offset % 32) == 0;
  if (P.decode_counts) ok = ok && aligned(P.decode_counts, 16) && (P.counts_stride % 4) == 0;
  if (P.context_counts) ok = ok && aligned(P.context_counts, 16) && (P.counts_stride % 4) == 0;
  if (P.bias) ok = ok && aligned(P.bias, 16) && (P.bias_stride % 8) == 0;
  return ok;
}

// bulk copies additionally read grammar words in 16-byte groups
static bool params_tma_ok(const SonicSamplingParams& P, int64_t shard_offset) {
  bool ok = params_vec_ok(P, shard_offset) && (shard_offset % 128) == 0;
  if (P.grammar) ok = ok && aligned(P.grammar, 16) && (P.grammar_stride % 4) == 0;
  return ok;
}

static sonic_status check_params(const SonicSamplingParams& P) {
  if (!P.indicators) return fail(SONIC_ERR_INVALID_ARGUMENT, "indicators must not be NULL");
  if (P.slot_mapping && P.slot_dtype != SONIC_DTYPE_I32 && P.slot_dtype != SONIC_DTYPE_I64)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "slot_mapping dtype must be i32 or i64");
  return SONIC_OK;
}

static Plan singular_plan(int64_t rows, int64_t V) { return split_plan(rows, V, CH); }
static Plan multistep_plan(int64_t rows, int64_t V) { return split_plan(rows, V, CH); }

static int64_t multistep_rows(const SonicMultistepArgs* a) {
  return a->total_rows > 0 ? a->total_rows : (int64_t)a->batch_size * (a->lookahead + 1);
}

}  // namespace sonic

using namespace sonic;

extern "C" {

int32_t sonic_abi_version(void) { return SONIC_B200_ABI_VERSION; }

const char* sonic_last_error(void) { return g_last_error.c_str(); }

size_t sonic_fused_singular_workspace_size(const SonicSingularArgs* a) {
  if (!a || a->rows <= 0 || a->vocab_size < kMaxK) return 0;
  return workspace_bytes(a->rows, a->rows, singular_plan(a->rows, a->vocab_size).splits);
}

size_t sonic_fused_multistep_workspace_size(const SonicMultistepArgs* a) {
  if (!a || a->batch_size <= 0 || a->vocab_size < kMaxK) return 0;
  return workspace_bytes(multistep_rows(a), a->batch_size, multistep_plan(multistep_rows(a), a->vocab_size).splits);
}

size_t sonic_bounded_topk_workspace_size(const SonicTopKArgs* a) {
  if (!a || a->rows <= 0 || a->vocab_size < kMaxK) return 0;
  return workspace_bytes(a->rows, a->rows, singular_plan(a->rows, a->vocab_size).splits);
}

}  // extern "C"

namespace sonic {

// Host checks shared by the singular entry points (selection arguments only when `selects`).
static sonic_status check_singular(const SonicSingularArgs* a, bool selects) {
  if (a->rows < 0 || a->rows > 65535) return fail(SONIC_ERR_INVALID_ARGUMENT, "rows must be in [0, 65535]");
  if (a->vocab_size < kMaxK) return fail(SONIC_ERR_INVALID_ARGUMENT, "vocab_size must be >= 128");
  if (sonic_status s = check_block_n(a->block_n)) return s;
  if (sonic_status s = check_params(a->params)) return s;
  if (!a->tokens) return fail(SONIC_ERR_INVALID_ARGUMENT, "tokens must not be NULL");
  if (a->lookahead < 0 || a->lookahead > SONIC_MAX_LOOKAHEAD)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "lookahead must be in [0, 15]");
  if (a->d2t && a->d2t_dtype != SONIC_DTYPE_I32 && a->d2t_dtype != SONIC_DTYPE_I64)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "d2t dtype must be i32 or i64");
  if (!selects) return SONIC_OK;
  if (!(a->flags & SONIC_FLAG_PHILOX) && !a->gumbel)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "gumbel noise must not be NULL without SONIC_FLAG_PHILOX");
  if ((a->flags & SONIC_FLAG_UPDATE_COUNTS) && !a->params.decode_counts)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "`update_counts` is True but `decode_counts` is None");
  if ((a->flags & SONIC_FLAG_PROBABILITIES) && a->probabilities && a->probabilities_dtype != SONIC_DTYPE_BF16 &&
      a->probabilities_dtype != SONIC_DTYPE_F32)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "probabilities dtype must be bf16 or f32");
  if (a->max_top_logprobs < 0 || a->max_top_logprobs > kMaxK)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "max_top_logprobs must be in [0, 128]");
  if (a->logprobs_dtype != SONIC_DTYPE_BF16 && a->logprobs_dtype != SONIC_DTYPE_F32)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logprobs dtype must be bf16 or f32");
  return SONIC_OK;
}

// The general kernel's splits: grids of several waves pay every CTA's fixed costs (row set-up,
// first-chunk latency, the split's end) once per CTA, so they take as few splits as keep the
// TARGET_CTAS slots busy, down to one CTA per row (at most SPLIT_MAX_COLS columns a CTA). Never
// more splits than the workspace was sized for (p.splits).
static Plan wave_plan(const Plan& p, int64_t rows, int64_t V) {
  if ((int64_t)p.splits * rows <= TARGET_CTAS) return p;
  int64_t sp = std::max<int64_t>(1, std::min<int64_t>(p.splits, TARGET_CTAS / std::max<int64_t>(1, rows)));
  sp = std::max<int64_t>(sp, (V + SPLIT_MAX_COLS - 1) / SPLIT_MAX_COLS);
  int64_t wc = (V + sp - 1) / sp;
  wc = (wc + CH - 1) / CH * CH;
  Plan w;
  w.splits = (int)((V + wc - 1) / wc);
  w.cols = (int)wc;
  return w;
}

// Rows with no per-column processor anywhere in the call stream through the logits-only
// kernel: the rows of a singular call, their vocab-sharded candidates (`cand`), or the rows of a
// multistep call (`ms`). `used` gets the column splits of the launch (at most p.splits, so
// the lists fit the workspace carved for p).
static cudaError_t plain_launch(const SonicSingularArgs& a, const Plan& p, const Workspace& ws, cudaStream_t st,
                                uint64_t* cand, const MsRows* ms, int& used) {
  const bool xvec = aligned(a.logits, 16) && (a.logits_stride % 8) == 0;
  const int pm = xvec ? kTma : kScalar;
  const bool pdl = (a.flags & SONIC_FLAG_PDL) != 0;
  const int l2 = ilog2(a.block_n);
  // a grid of several waves keeps 4 CTAs an SM busy with a 3-stage ring (their fixed costs
  // overlap); one wave streams longer rows per CTA and takes 3 CTAs with a deeper ring
  const bool waves = (int64_t)p.splits * a.rows > TARGET_CTAS;
  const int nst = waves ? PNST_WAVES : PNST_ONE;
  const size_t ring = (size_t)nst * PSTAGE;
  // Grids of several waves pay every CTA's fixed costs (final absorbs, fold, list, ticket,
  // merge) once per CTA: they take as few CTAs as keep the SMs' 4 slots busy, down to one
  // CTA per row, which then needs no merge at all (a CTA covers up to PLAIN_MAX_COLS
  // columns). Never more splits than the workspace was sized for.
  Plan wp = p;
  if (waves && pm == kTma) {
    int64_t sp = std::max<int64_t>(1, std::min<int64_t>(p.splits, PLAIN_SLOTS / std::max<int64_t>(1, a.rows)));
    sp = std::max<int64_t>(sp, (a.vocab_size + PLAIN_MAX_COLS - 1) / PLAIN_MAX_COLS);
    int64_t wc = (a.vocab_size + sp - 1) / sp;
    wc = (wc + PCH - 1) / PCH * PCH;
    wp.splits = (int)((a.vocab_size + wc - 1) / wc);
    wp.cols = (int)wc;
  }
  used = wp.splits;
  const dim3 grid(wp.splits, a.rows);
  const MsRows m = ms ? *ms : MsRows{nullptr, nullptr, 0, 0};
  auto go = [&](auto msc) {
    constexpr bool M = decltype(msc)::value;
    if (pm != kTma) return launch(plain_kernel<kScalar, 3, M>, grid, 0, st, pdl, a, wp.splits, wp.cols, l2, ws, 0, cand, m);
    if (waves) return launch(plain_kernel<kTma, 4, M>, grid, ring, st, pdl, a, wp.splits, wp.cols, l2, ws, nst, cand, m);
    return launch(plain_kernel<kTma, 3, M>, grid, ring, st, pdl, a, wp.splits, wp.cols, l2, ws, nst, cand, m);
  };
  return ms ? go(std::true_type{}) : go(std::false_type{});
}

// The singular launch; with `cand` the last CTA of a row writes the row's top-128 keys
// (global columns) there instead of selecting.
static sonic_status singular_launch(const SonicSingularArgs* a, void* stream, uint64_t* cand, const char* what) {
  if (!a->logits || a->logits_dtype != SONIC_DTYPE_BF16)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logits must be a non-NULL bf16 tensor");
  const Plan p = singular_plan(a->rows, a->vocab_size);
  const size_t need = workspace_bytes(a->rows, a->rows, p.splits);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(SONIC_ERR_WORKSPACE, "workspace smaller than sonic_fused_singular_workspace_size()");
  const Workspace ws = carve(a->workspace, a->rows, a->rows, p.splits);
  const bool xvec = aligned(a->logits, 16) && (a->logits_stride % 8) == 0;
  const bool ind = a->d2t != nullptr;
  const SonicSamplingParams& P = a->params;
  if (!ind && !P.grammar && !P.decode_counts && !P.context_counts && !P.bias) {
    // no per-column processor anywhere in the call: logits-only streaming kernel (also for
    // the vocab-sharded candidates, `cand`)
    int used = 0;
    return check_launch(plain_launch(*a, p, ws, (cudaStream_t)stream, cand, nullptr, used), what);
  }
  int mode = (xvec && (ind || params_vec_ok(a->params, a->shard_offset))) ? kVec : kScalar;
  // with a d2t table the ring streams the logits only, which xvec already allows
  if (mode == kVec && (ind || params_tma_ok(a->params, a->shard_offset))) mode = kTma;
  // ring grids of several waves: one CTA per row where the row fits (wide keys)
  const Plan wp = mode == kTma ? wave_plan(p, a->rows, a->vocab_size) : p;
  const bool wide = wp.cols > MAX_SPLIT_COLS;
  dim3 grid(wp.splits, a->rows);
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = (a->flags & SONIC_FLAG_PDL) != 0;
  const int l2 = ilog2(a->block_n);
  const size_t ring = mode == kTma ? (size_t)RING_BYTES : 0;
  const int sp = wp.splits, sc = wp.cols;
  cudaError_t e;
  if (ind)
    e = mode == kTma
            ? (wide ? launch(singular_kernel<kTma, true, false, true>, grid, ring, st, pdl, *a, sp, sc, l2, ws, cand, MsRows{})
                    : launch(singular_kernel<kTma, true, false>, grid, ring, st, pdl, *a, sp, sc, l2, ws, cand, MsRows{}))
        : mode == kVec ? launch(singular_kernel<kVec, true, false>, grid, 0, st, pdl, *a, sp, sc, l2, ws, cand, MsRows{})
                       : launch(singular_kernel<kScalar, true, false>, grid, 0, st, pdl, *a, sp, sc, l2, ws, cand, MsRows{});
  else if (mode == kTma)
    e = wide ? launch(singular_kernel<kTma, false, false, true>, grid, ring, st, pdl, *a, sp, sc, l2, ws, cand, MsRows{})
             : launch(singular_kernel<kTma, false, false>, grid, ring, st, pdl, *a, sp, sc, l2, ws, cand, MsRows{});
  else
    e = mode == kVec ? launch(singular_kernel<kVec, false, false>, grid, 0, st, pdl, *a, sp, sc, l2, ws, cand, MsRows{})
                     : launch(singular_kernel<kScalar, false, false>, grid, 0, st, pdl, *a, sp, sc, l2, ws, cand, MsRows{});
  return check_launch(e, what);
}

}  // namespace sonic

extern "C" {

sonic_status sonic_fused_singular(const SonicSingularArgs* a, void* stream) {
  if (!a) return fail(SONIC_ERR_INVALID_ARGUMENT, "args must not be NULL");
  if (a->rows == 0) return SONIC_OK;
  if (sonic_status s = check_singular(a, true)) return s;
  return singular_launch(a, stream, nullptr, "sonic_fused_singular");
}

sonic_status sonic_shard_candidates(const SonicSingularArgs* a, uint64_t* keys, void* stream) {
  if (!a) return fail(SONIC_ERR_INVALID_ARGUMENT, "args must not be NULL");
  if (a->rows == 0) return SONIC_OK;
  if (!keys) return fail(SONIC_ERR_INVALID_ARGUMENT, "keys must not be NULL");
  if (sonic_status s = check_singular(a, false)) return s;
  return singular_launch(a, stream, keys, "sonic_shard_candidates");
}

sonic_status sonic_merge_candidates(const SonicSingularArgs* a, const uint64_t* gathered, int32_t world,
                                    void* stream) {
  if (!a) return fail(SONIC_ERR_INVALID_ARGUMENT, "args must not be NULL");
  if (a->rows == 0) return SONIC_OK;
  if (!gathered) return fail(SONIC_ERR_INVALID_ARGUMENT, "gathered keys must not be NULL");
  if (world < 1 || world > MAX_SPLITS) return fail(SONIC_ERR_INVALID_ARGUMENT, "world must be in [1, 32]");
  if (sonic_status s = check_singular(a, true)) return s;
  const bool pdl = (a->flags & SONIC_FLAG_PDL) != 0;
  const cudaError_t e = launch(merge_candidates_kernel, dim3(a->rows), 0, (cudaStream_t)stream, pdl, *a, gathered,
                               (int)world);
  return check_launch(e, "sonic_merge_candidates");
}


sonic_status sonic_bounded_topk(const SonicTopKArgs* a, void* stream) {
  if (!a) return fail(SONIC_ERR_INVALID_ARGUMENT, "args must not be NULL");
  if (a->rows == 0) return SONIC_OK;
  if (a->rows < 0 || a->rows > 65535) return fail(SONIC_ERR_INVALID_ARGUMENT, "rows must be in [0, 65535]");
  if (a->vocab_size < kMaxK) return fail(SONIC_ERR_INVALID_ARGUMENT, "vocab_size must be >= 128");
  if (a->k < 1 || a->k > kMaxK || (a->k & (a->k - 1)))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "k must be a power of two in [1, 128]");
  if (!a->logits || (a->logits_dtype != SONIC_DTYPE_BF16 && a->logits_dtype != SONIC_DTYPE_F32))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logits must be a non-NULL bf16 or f32 tensor");
  if (!a->values || (a->values_dtype != SONIC_DTYPE_BF16 && a->values_dtype != SONIC_DTYPE_F32))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "values must be a non-NULL bf16 or f32 tensor");
  if (!a->indices || (a->indices_dtype != SONIC_DTYPE_I32 && a->indices_dtype != SONIC_DTYPE_I64))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "indices must be a non-NULL i32 or i64 tensor");
  const Plan p = singular_plan(a->rows, a->vocab_size);
  const size_t need = workspace_bytes(a->rows, a->rows, p.splits);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(SONIC_ERR_WORKSPACE, "workspace smaller than sonic_bounded_topk_workspace_size()");
  const Workspace ws = carve(a->workspace, a->rows, a->rows, p.splits);
  const bool f32 = a->logits_dtype == SONIC_DTYPE_F32;
  const bool vec = aligned(a->logits, 16) && (a->logits_stride % (f32 ? 4 : 8)) == 0;
  dim3 grid(p.splits, a->rows);
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = (a->flags & SONIC_FLAG_PDL) != 0;
  cudaError_t e;
  if (f32)
    e = vec ? launch(topk_kernel<kVec, true>, grid, 0, st, pdl, *a, p.splits, p.cols, ws)
            : launch(topk_kernel<kScalar, true>, grid, 0, st, pdl, *a, p.splits, p.cols, ws);
  else
    e = vec ? launch(topk_kernel<kVec, false>, grid, 0, st, pdl, *a, p.splits, p.cols, ws)
            : launch(topk_kernel<kScalar, false>, grid, 0, st, pdl, *a, p.splits, p.cols, ws);
  return check_launch(e, "sonic_bounded_topk");
}

sonic_status sonic_fused_multistep(const SonicMultistepArgs* a, void* stream) {
  if (!a) return fail(SONIC_ERR_INVALID_ARGUMENT, "args must not be NULL");
  if (a->batch_size == 0) return SONIC_OK;
  if (a->batch_size < 0 || a->batch_size > 65535)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "batch_size must be in [0, 65535]");
  if (a->vocab_size < kMaxK) return fail(SONIC_ERR_INVALID_ARGUMENT, "vocab_size must be >= 128");
  if (a->lookahead < 1 || a->lookahead > SONIC_MAX_LOOKAHEAD)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "lookahead must be in [1, 15]");
  if (sonic_status s = check_block_n(a->block_n)) return s;
  if (sonic_status s = check_params(a->params)) return s;
  if (!a->logits || a->logits_dtype != SONIC_DTYPE_BF16)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logits must be a non-NULL bf16 tensor");
  if (!a->drafted_tokens || !a->tokens || !a->offsets)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "drafted_tokens, tokens and offsets must not be NULL");
  if (!(a->flags & SONIC_FLAG_PHILOX) && (!a->gumbel || !a->uniform))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "gumbel and uniform noise must not be NULL without SONIC_FLAG_PHILOX");
  if (a->draft_probs && a->draft_dtype != SONIC_DTYPE_F32 && a->draft_dtype != SONIC_DTYPE_BF16)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "draft probabilities dtype must be f32 or bf16");
  if ((a->flags & SONIC_FLAG_UPDATE_COUNTS) && !a->params.decode_counts)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "`update_counts` is True but `decode_counts` is None");
  if (a->max_top_logprobs < 0 || a->max_top_logprobs > kMaxK)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "max_top_logprobs must be in [0, 128]");
  if (a->logprobs_dtype != SONIC_DTYPE_BF16 && a->logprobs_dtype != SONIC_DTYPE_F32)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logprobs dtype must be bf16 or f32");
  const int64_t rows = multistep_rows(a);
  if (rows > 65535) return fail(SONIC_ERR_INVALID_ARGUMENT, "multistep rows (batch x steps) must be <= 65535");
  const Plan p = multistep_plan(rows, a->vocab_size);
  const size_t need = workspace_bytes(rows, a->batch_size, p.splits);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(SONIC_ERR_WORKSPACE, "workspace smaller than sonic_fused_multistep_workspace_size()");
  const Workspace ws = carve(a->workspace, rows, a->batch_size, p.splits);
  // the rows stream through the singular kernel (MS mode), which reads these fields only
  SonicSingularArgs sa;
  memset(&sa, 0, sizeof(sa));
  sa.rows = (int32_t)rows;
  sa.vocab_size = a->vocab_size;
  sa.block_n = a->block_n;
  sa.shard_offset = a->shard_offset;
  sa.flags = a->flags & (SONIC_FLAG_PDL | SONIC_FLAG_DEBUG_STALL_RING);
  sa.logits = a->logits;
  sa.logits_dtype = a->logits_dtype;
  sa.logits_stride = a->logits_stride;
  sa.params = a->params;
  sa.tokens = a->tokens;
  const MsRows m{a->cu_seqlens, a->drafted_tokens, a->batch_size, a->lookahead};
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = (a->flags & SONIC_FLAG_PDL) != 0;
  const int l2 = ilog2(a->block_n);
  const SonicSamplingParams& P = a->params;
  if (!P.grammar && !P.decode_counts && !P.context_counts && !P.bias) {
    // no per-column processor anywhere in the call: the rows stream through the logits-only
    // kernel, whose column splits the verification then reads
    int used = 0;
    if (sonic_status s = check_launch(plain_launch(sa, p, ws, st, nullptr, &m, used), "sonic_fused_multistep (rows)"))
      return s;
    return check_launch(launch(ms_verify_kernel, dim3(a->batch_size), 0, st, pdl, *a, used, l2, ws),
                        "sonic_fused_multistep");
  }
  const bool xvec = aligned(a->logits, 16) && (a->logits_stride % 8) == 0;
  int mode = (xvec && params_vec_ok(a->params, a->shard_offset)) ? kVec : kScalar;
  if (mode == kVec && params_tma_ok(a->params, a->shard_offset)) mode = kTma;
  const Plan wp = mode == kTma ? wave_plan(p, rows, a->vocab_size) : p;
  const bool wide = wp.cols > MAX_SPLIT_COLS;
  const dim3 grid(wp.splits, (unsigned)rows);
  cudaError_t e;
  if (mode == kTma)
    e = wide ? launch(singular_kernel<kTma, false, true, true>, grid, (size_t)RING_BYTES, st, pdl, sa, wp.splits, wp.cols,
                      l2, ws, (uint64_t*)nullptr, m)
             : launch(singular_kernel<kTma, false, true>, grid, (size_t)RING_BYTES, st, pdl, sa, wp.splits, wp.cols, l2,
                      ws, (uint64_t*)nullptr, m);
  else if (mode == kVec)
    e = launch(singular_kernel<kVec, false, true>, grid, 0, st, pdl, sa, wp.splits, wp.cols, l2, ws, (uint64_t*)nullptr, m);
  else
    e = launch(singular_kernel<kScalar, false, true>, grid, 0, st, pdl, sa, wp.splits, wp.cols, l2, ws,
               (uint64_t*)nullptr, m);
  if (sonic_status s = check_launch(e, "sonic_fused_multistep (rows)")) return s;
  e = launch(ms_verify_kernel, dim3(a->batch_size), 0, st, pdl, *a, wp.splits, l2, ws);
  return check_launch(e, "sonic_fused_multistep");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// noise staging (ops/copy.py:21-127 indexed_copy): the rows of `source` named by `indices`
// whose indicator lacks the greedy bit are copied to the same rows of `target`
//
// A pure HBM stream (read + write once). Each CTA is one issuing thread driving a ring of
// 16 KB 1-D bulk copies: global -> shared on an mbarrier, then shared -> global as a bulk
// store; a stage is refilled once its store has read it (wait_group.read). The CTA's chunks
// are a contiguous run of the selected rows' 16 KB chunks. Rows whose bytes, base addresses
// or stride are not 16-byte multiples take an element-wise kernel instead.
// ---------------------------------------------------------------------------------------

namespace sonic {

constexpr int CP_CHUNK = 16384;  // bytes of one bulk copy
constexpr int CP_STAGES = 4;     // 64 KB of ring: 3 CTAs an SM
constexpr int CP_CTAS_PER_SM = 3;

struct CopyArgs {
  const unsigned char* src;
  unsigned char* dst;
  int64_t stride;  // bytes between rows (source and target alike)
  int64_t row;     // bytes copied per row
  const void* indices;
  int32_t index_dtype;
  int32_t count;
  const uint16_t* indicator;
  int64_t rows;  // rows of source / target: other indices are skipped
};

__device__ __forceinline__ void bulk_store(void* gdst, const void* ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_addr(ssrc)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// every committed bulk store has finished reading its shared memory
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// every committed bulk store has completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__global__ void __launch_bounds__(32) indexed_copy_kernel(const CopyArgs c, int64_t chunks_per_row, int64_t total) {
  extern __shared__ __align__(128) unsigned char ring[];
  __shared__ uint64_t bars[CP_STAGES];
  if (threadIdx.x != 0) return;
  const int64_t G = gridDim.x;
  const int64_t q0 = (int64_t)blockIdx.x * total / G;
  const int64_t n = ((int64_t)blockIdx.x + 1) * total / G - q0;
  for (int i = 0; i < CP_STAGES; ++i) mbar_init(&bars[i], 1);
  mbar_fence_init();
  unsigned char* dst[CP_STAGES];
  uint32_t bytes[CP_STAGES];
  uint32_t live = 0;  // stages holding a chunk to store
  // chunk j of this CTA into stage j % CP_STAGES: a bulk load, or a plain arrival for a
  // chunk of a greedy row (nothing to copy), so that every stage completes once per use
  auto issue = [&](int64_t j) {
    const int s = (int)(j % CP_STAGES);
    const int64_t q = q0 + j;
    const int64_t i = q / chunks_per_row, piece = q % chunks_per_row;
    const int64_t r = load_index(c.indices, c.index_dtype, i);
    if (r < 0 || r >= c.rows || (c.indicator[r] & 0x40)) {
      live &= ~(1u << s);
      mbar_arrive(&bars[s]);
      return;
    }
    const int64_t off = r * c.stride + piece * CP_CHUNK;
    const uint32_t nb = (uint32_t)min((int64_t)CP_CHUNK, c.row - piece * CP_CHUNK);
    live |= 1u << s;
    dst[s] = c.dst + off;
    bytes[s] = nb;
    mbar_expect_tx(&bars[s], nb);
    bulk_load(ring + s * CP_CHUNK, c.src + off, nb, &bars[s]);
  };
  for (int64_t j = 0; j < min(n, (int64_t)CP_STAGES); ++j) issue(j);
  for (int64_t j = 0; j < n; ++j) {
    const int s = (int)(j % CP_STAGES);
    if (!mbar_wait_bounded(&bars[s], (uint32_t)((j / CP_STAGES) & 1), WAIT_LIMIT)) {
      // the chunk never landed: store nothing more, record the error in the library's word
      // (sonic_workspace_error(NULL, ...)), and let the copies in flight land before leaving
      atomicOr(reinterpret_cast<uint32_t*>(g_static_scratch), (uint32_t)SONIC_DEVICE_ERR_WAIT);
      for (int64_t jj = j; jj < min(n, j + (int64_t)CP_STAGES); ++jj)
        mbar_wait_bounded(&bars[jj % CP_STAGES], (uint32_t)((jj / CP_STAGES) & 1), WAIT_LIMIT);
      break;
    }
    if ((live >> s) & 1u) {
      bulk_store(dst[s], ring + s * CP_CHUNK, bytes[s]);
      bulk_commit();
    }
    if (j + CP_STAGES < n) {
      bulk_wait_read_all();  // the store just issued from stage s has read it
      issue(j + CP_STAGES);
    }
  }
  bulk_wait_all();
}

// the same copy element by element (rows not in 16-byte units)
template <typename E>
__global__ void __launch_bounds__(256) indexed_copy_elems(const CopyArgs c, int64_t elems) {
  for (int64_t i = blockIdx.y; i < c.count; i += gridDim.y) {
    const int64_t r = load_index(c.indices, c.index_dtype, i);
    if (r < 0 || r >= c.rows || (c.indicator[r] & 0x40)) continue;
    const E* src = reinterpret_cast<const E*>(c.src + r * c.stride);
    E* dst = reinterpret_cast<E*>(c.dst + r * c.stride);
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < elems; e += (int64_t)gridDim.x * blockDim.x)
      __stcs(dst + e, __ldcs(src + e));
  }
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return n > 0 ? n : 148;
}

// ---------------------------------------------------------------------------------------
// batched slot population (core/buffer.py:1026-1352: step_grammar, update, allocate)
//
// CTA (x, i) owns columns [x * POP_RANGE, +POP_RANGE) of call slot i's rows. The row parts
// are built in shared memory (prompt histogram, bias row) or copied, and every destination
// byte is written once with 16-byte stores where the row allows. A prompt of L tokens is
// scanned by each of the slot's ceil(V / POP_RANGE) CTAs (from L2); every CTA counts only
// its own columns, so no global atomics and no ordering between CTAs are needed.
// ---------------------------------------------------------------------------------------

constexpr int POP_RANGE = 4096;  // columns of one CTA
constexpr int POP_NT = 256;
constexpr int POP_UNROLL = 8;  // prompt ids a thread loads before counting them

// n int32 from shared memory (or zeros when src is NULL) to dst
__device__ __forceinline__ void pop_store_i32(int32_t* dst, const int32_t* src, int n) {
  int i0 = 0;
  if (((uintptr_t)dst & 15) == 0) {
    const int n4 = n >> 2;
    for (int v = threadIdx.x; v < n4; v += POP_NT)
      reinterpret_cast<int4*>(dst)[v] = src ? reinterpret_cast<const int4*>(src)[v] : make_int4(0, 0, 0, 0);
    i0 = n4 << 2;
  }
  for (int e = i0 + threadIdx.x; e < n; e += POP_NT) dst[e] = src ? src[e] : 0;
}

// n int32 global to global
__device__ __forceinline__ void pop_copy_i32(int32_t* dst, const int32_t* src, int n) {
  int i0 = 0;
  if ((((uintptr_t)dst | (uintptr_t)src) & 15) == 0) {
    const int n4 = n >> 2;
    for (int v = threadIdx.x; v < n4; v += POP_NT)
      reinterpret_cast<int4*>(dst)[v] = __ldcs(reinterpret_cast<const int4*>(src) + v);
    i0 = n4 << 2;
  }
  for (int e = i0 + threadIdx.x; e < n; e += POP_NT) dst[e] = __ldcs(src + e);
}

__global__ void __launch_bounds__(POP_NT) populate_kernel(const SonicPopulateArgs a) {
  __shared__ __align__(16) int32_t hist[POP_RANGE];
  __shared__ __align__(16) uint16_t brow[POP_RANGE];
  const int tid = threadIdx.x;
  const int i = blockIdx.y;
  const int64_t V = a.vocab_size;
  const int64_t c0 = (int64_t)blockIdx.x * POP_RANGE;
  const int n = (int)min((int64_t)POP_RANGE, V - c0);  // > 0: the grid covers V exactly
  const bool hist_on = (a.parts & SONIC_POPULATE_HISTOGRAM) != 0;
  const bool dense_on = !hist_on && (a.parts & SONIC_POPULATE_DENSE_COUNTS) != 0;
  const bool bias_on = (a.parts & SONIC_POPULATE_BIAS) != 0;
  const bool gram_on = (a.parts & SONIC_POPULATE_GRAMMAR) != 0;

  // first round trip: every per-slot offset, loaded together
  const int64_t slot = a.positions[i];
  int64_t t0 = 0, t1 = 0, b0 = 0, b1 = 0;
  int64_t grow = -1;
  int gsteps = 0;
  if (hist_on) {
    t0 = a.token_offsets[i];
    t1 = a.token_offsets[i + 1];
  }
  if (bias_on && a.bias_offsets) {
    b0 = a.bias_offsets[i];
    b1 = a.bias_offsets[i + 1];
  }
  if (gram_on) {
    grow = a.grammar_rows[i];
    gsteps = a.grammar_steps[i];
  }
  if (slot < 0 || slot >= a.num_slots) return;  // the host checks positions; never write outside

  if ((a.parts & SONIC_POPULATE_SCALARS) && blockIdx.x == 0 && tid < 10) {
    // PinnedRelay.populate / RepetitionPenalties.populate / Flags.update + transfer
    const uint16_t* f = a.values_bf16 + (int64_t)i * 6;
    switch (tid) {
      case 0: a.temperature[slot] = f[0]; break;
      case 1: a.top_p[slot] = f[1]; break;
      case 2: a.min_p[slot] = f[2]; break;
      case 3: a.multiplicative[slot] = f[3]; break;
      case 4: a.frequency[slot] = f[4]; break;
      case 5: a.presence[slot] = f[5]; break;
      case 6: a.top_k[slot] = a.values_i32[(int64_t)i * 2]; break;
      case 7: a.top_logprobs[slot] = a.values_i32[(int64_t)i * 2 + 1]; break;
      case 8: a.flags_target[slot] = a.indicators[(int64_t)i * 2]; break;
      default: a.flags_draft[slot] = a.indicators[(int64_t)i * 2 + 1]; break;
    }
  }

  int32_t* ctx = a.context_counts + slot * a.counts_stride + c0;
  int32_t* dec = a.decode_counts + slot * a.counts_stride + c0;
  if (hist_on) {
    pop_store_i32(dec, nullptr, n);  // TokenCounts.allocate: decode = 0, no dependency
  } else if (dense_on) {
    // TokenCounts.update: both rows copied
    pop_copy_i32(ctx, a.dense_context + (int64_t)i * V + c0, n);
    pop_copy_i32(dec, a.dense_decode + (int64_t)i * V + c0, n);
  }

  // second round trip: the first prompt ids, bias entry and bitmask word of this thread,
  // issued together before the shared-memory rows are zeroed
  int32_t tk[POP_UNROLL];
#pragma unroll
  for (int k = 0; k < POP_UNROLL; ++k) {
    const int64_t t = t0 + k * POP_NT + tid;
    tk[k] = t < t1 ? __ldg(a.tokens + t) : -1;
  }
  int32_t btok = -1;
  uint16_t bval = 0;
  if (b0 + tid < b1) {
    btok = __ldg(a.bias_tokens + b0 + tid);
    bval = __ldg(a.bias_values + b0 + tid);
  }
  const int64_t W = (V + 31) / 32;
  const int64_t w0 = c0 / 32;
  const int nw = (int)min((int64_t)(POP_RANGE / 32), W - w0);
  uint32_t gword = 0;
  if (grow >= 0 && tid < nw) gword = __ldg(a.grammar_words + grow * W + w0 + tid);

  if (hist_on || bias_on) {
    if (hist_on)
      for (int e = tid; e < POP_RANGE / 4; e += POP_NT) reinterpret_cast<int4*>(hist)[e] = make_int4(0, 0, 0, 0);
    if (bias_on)
      for (int e = tid; e < POP_RANGE / 8; e += POP_NT) reinterpret_cast<uint4*>(brow)[e] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    if (hist_on) {
      // TokenCounts.populate: scatter_add of ones at the prompt's ids in this CTA's columns,
      // POP_UNROLL independent loads a thread ahead of their shared-memory atomics
      for (int64_t base = t0;;) {
#pragma unroll
        for (int k = 0; k < POP_UNROLL; ++k)
          if (tk[k] >= c0 && tk[k] < c0 + n) atomicAdd(&hist[tk[k] - c0], 1);
        base += (int64_t)POP_NT * POP_UNROLL;
        if (base >= t1) break;
#pragma unroll
        for (int k = 0; k < POP_UNROLL; ++k) {
          const int64_t t = base + k * POP_NT + tid;
          tk[k] = t < t1 ? __ldg(a.tokens + t) : -1;
        }
      }
    }
    if (bias_on) {
      // PinnedRelay.update_bias: the slot's entries land on the zeroed row
      if (btok >= c0 && btok < c0 + n) brow[btok - c0] = bval;
      for (int64_t t = b0 + POP_NT + tid; t < b1; t += POP_NT) {
        const int64_t tok = a.bias_tokens[t];
        if (tok >= c0 && tok < c0 + n) brow[tok - c0] = a.bias_values[t];
      }
    }
    __syncthreads();
    if (hist_on) pop_store_i32(ctx, hist, n);
    if (bias_on) {
      uint16_t* dst = a.bias + slot * a.bias_stride + c0;
      int e0 = 0;
      if (((uintptr_t)dst & 15) == 0) {
        const int n8 = n >> 3;
        for (int v = tid; v < n8; v += POP_NT) reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(brow)[v];
        e0 = n8 << 3;
      }
      for (int e = e0 + tid; e < n; e += POP_NT) dst[e] = brow[e];
    }
  }

  if (grow >= 0 && tid < nw) {
    // step_grammar: grammar[slot, step] (admission) or grammar[slot] (every step, one row
    // broadcast or one row a step) = the bitmask
    const int s0 = a.grammar_step >= 0 ? a.grammar_step : 0;
    const int s1 = a.grammar_step >= 0 ? a.grammar_step + 1 : a.timesteps;
    uint32_t* dst = a.grammar + slot * a.grammar_slot_stride + w0 + tid;
    for (int s = s0; s < s1; ++s) {
      const uint32_t w = (gsteps > 1 && s > s0) ? __ldg(a.grammar_words + (grow + (s - s0)) * W + w0 + tid) : gword;
      dst[(int64_t)s * a.grammar_step_stride] = w;
    }
  }
}

}  // namespace sonic

extern "C" {

sonic_status sonic_indexed_copy(const void* source, void* target, int64_t rows, int64_t stride, int64_t cols,
                                int32_t elem_bytes, const void* indices, int32_t index_dtype, int32_t count,
                                const uint16_t* indicator, void* stream) {
  if (count < 0 || cols < 0 || stride < 0 || rows < 0)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "rows, count, cols and stride must be >= 0");
  if (count == 0 || cols == 0 || rows == 0) return SONIC_OK;
  if (!source || !target || !indices || !indicator)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "source, target, indices and indicator must not be NULL");
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "elem_bytes must be 1, 2, 4 or 8");
  if (index_dtype != SONIC_DTYPE_I32 && index_dtype != SONIC_DTYPE_I64)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "indices dtype must be i32 or i64");
  if (cols > stride) return fail(SONIC_ERR_INVALID_ARGUMENT, "cols must not exceed the row stride");
  CopyArgs c;
  c.src = (const unsigned char*)source;
  c.dst = (unsigned char*)target;
  c.stride = stride * elem_bytes;
  c.row = cols * elem_bytes;
  c.indices = indices;
  c.index_dtype = index_dtype;
  c.count = count;
  c.indicator = indicator;
  c.rows = rows;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e;
  if (aligned(source, 16) && aligned(target, 16) && c.stride % 16 == 0 && c.row % 16 == 0) {
    const int64_t cpr = (c.row + CP_CHUNK - 1) / CP_CHUNK;
    const int64_t total = cpr * count;
    const int64_t grid = std::min<int64_t>(total, (int64_t)sm_count() * CP_CTAS_PER_SM);
    const size_t smem = (size_t)CP_STAGES * CP_CHUNK;
    e = cudaFuncSetAttribute(indexed_copy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) {
      indexed_copy_kernel<<<dim3((unsigned)grid), dim3(32), smem, st>>>(c, cpr, total);
      e = cudaGetLastError();
    }
  } else {
    const dim3 grid((unsigned)std::min<int64_t>((cols + 255) / 256, 64), (unsigned)std::min<int64_t>(count, 65535));
    switch (elem_bytes) {
      case 1: indexed_copy_elems<uint8_t><<<grid, 256, 0, st>>>(c, cols); break;
      case 2: indexed_copy_elems<uint16_t><<<grid, 256, 0, st>>>(c, cols); break;
      case 4: indexed_copy_elems<uint32_t><<<grid, 256, 0, st>>>(c, cols); break;
      default: indexed_copy_elems<unsigned long long><<<grid, 256, 0, st>>>(c, cols); break;
    }
    e = cudaGetLastError();
  }
  return check_launch(e, "sonic_indexed_copy");
}

sonic_status sonic_populate_slots(const SonicPopulateArgs* a, void* stream) {
  if (!a) return fail(SONIC_ERR_INVALID_ARGUMENT, "args must not be NULL");
  if (a->count < 0) return fail(SONIC_ERR_INVALID_ARGUMENT, "count must be >= 0");
  if (a->count == 0 || a->parts == 0) return SONIC_OK;
  constexpr uint32_t all = SONIC_POPULATE_SCALARS | SONIC_POPULATE_HISTOGRAM | SONIC_POPULATE_DENSE_COUNTS |
                           SONIC_POPULATE_BIAS | SONIC_POPULATE_GRAMMAR;
  if (a->parts & ~all) return fail(SONIC_ERR_INVALID_ARGUMENT, "unknown SONIC_POPULATE_* bits");
  if ((a->parts & SONIC_POPULATE_HISTOGRAM) && (a->parts & SONIC_POPULATE_DENSE_COUNTS))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "HISTOGRAM and DENSE_COUNTS are exclusive");
  if (a->count > 65535) return fail(SONIC_ERR_INVALID_ARGUMENT, "count must be <= 65535");
  if (a->num_slots <= 0 || a->vocab_size <= 0 || !a->positions)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "num_slots and vocab_size must be > 0 and positions non-NULL");
  if ((a->parts & SONIC_POPULATE_SCALARS) &&
      (!a->values_bf16 || !a->values_i32 || !a->indicators || !a->temperature || !a->top_p || !a->min_p ||
       !a->top_k || !a->top_logprobs || !a->multiplicative || !a->frequency || !a->presence || !a->flags_target ||
       !a->flags_draft))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "SCALARS needs every value and destination pointer");
  const bool counts = (a->parts & (SONIC_POPULATE_HISTOGRAM | SONIC_POPULATE_DENSE_COUNTS)) != 0;
  if (counts && (!a->context_counts || !a->decode_counts || a->counts_stride < a->vocab_size))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "count rows need both destinations and counts_stride >= vocab_size");
  if ((a->parts & SONIC_POPULATE_HISTOGRAM) && (!a->token_offsets || !a->tokens))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "HISTOGRAM needs token_offsets and tokens");
  if ((a->parts & SONIC_POPULATE_DENSE_COUNTS) && (!a->dense_context || !a->dense_decode))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "DENSE_COUNTS needs dense_context and dense_decode");
  if ((a->parts & SONIC_POPULATE_BIAS) &&
      (!a->bias || a->bias_stride < a->vocab_size || (a->bias_offsets && (!a->bias_tokens || !a->bias_values))))
    return fail(SONIC_ERR_INVALID_ARGUMENT, "BIAS needs the bias rows (bias_stride >= vocab_size) and its entries");
  if (a->parts & SONIC_POPULATE_GRAMMAR) {
    if (!a->grammar || !a->grammar_rows || !a->grammar_steps || !a->grammar_words || a->timesteps < 1)
      return fail(SONIC_ERR_INVALID_ARGUMENT, "GRAMMAR needs the grammar buffer, its rows and timesteps >= 1");
    if (a->grammar_step < -1 || a->grammar_step >= a->timesteps)
      return fail(SONIC_ERR_INVALID_ARGUMENT, "grammar_step must be -1 or in [0, timesteps)");
    const int64_t W = (a->vocab_size + 31) / 32;
    if (a->grammar_step_stride < W || a->grammar_slot_stride < (int64_t)(a->timesteps - 1) * a->grammar_step_stride + W)
      return fail(SONIC_ERR_INVALID_ARGUMENT, "grammar strides smaller than a row of ceil(vocab_size / 32) words");
  }
  const bool rows = counts || (a->parts & (SONIC_POPULATE_BIAS | SONIC_POPULATE_GRAMMAR));
  const int64_t gx = rows ? (a->vocab_size + POP_RANGE - 1) / POP_RANGE : 1;
  if (gx > 65535) return fail(SONIC_ERR_INVALID_ARGUMENT, "vocab_size too large");
  populate_kernel<<<dim3((unsigned)gx, (unsigned)a->count), dim3(POP_NT), 0, (cudaStream_t)stream>>>(*a);
  return check_launch(cudaGetLastError(), "sonic_populate_slots");
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// singular call without a caller workspace
//
// For hosts that cannot allocate device memory for this library: a serving engine that has
// already handed all free HBM to its KV cache, a foreign-language binding (cgo, JNI) with no
// access to the framework's caching allocator, or a latency-critical loop where a
// cudaMalloc, which may synchronise the device, is not acceptable. The scratch lives in a
// fixed device array instead; every GPU that loads this library holds it until the process
// exits.
// ---------------------------------------------------------------------------------------

namespace sonic {

constexpr int kMaxDevices = 64;

// Device address of g_static_scratch on the current device. In host code the array's name
// is only a host-side stand-in, so the address comes from cudaGetSymbolAddress, once per
// device, with that device current.
static sonic_status static_scratch(void** out) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(SONIC_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(SONIC_ERR_UNSUPPORTED, "device ordinal beyond the static scratch table");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return fail(SONIC_ERR_CUDA, std::string("cudaGetSymbolAddress(static scratch): ") + cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return SONIC_OK;
}

}  // namespace sonic

#ifdef SONIC_PHASE_STAMPS
// Diagnostic build only: copy the phase stamps to `host` (at most `bytes`) and, with `clear`,
// zero them on the device.
extern "C" sonic_status sonic_phase_stamps(void* host, size_t bytes, int32_t clear) {
  const size_t n = std::min(bytes, sizeof(PhaseStamps));
  if (host && n) {
    const cudaError_t e = cudaMemcpyFromSymbol(host, g_phase, n);
    if (e != cudaSuccess) return fail(SONIC_ERR_CUDA, std::string("phase stamps: ") + cudaGetErrorString(e));
  }
  if (clear) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_phase);
    if (e == cudaSuccess) e = cudaMemset(p, 0, sizeof(PhaseStamps));
    if (e != cudaSuccess) return fail(SONIC_ERR_CUDA, std::string("phase stamps: ") + cudaGetErrorString(e));
  }
  return SONIC_OK;
}
#endif

extern "C" sonic_status sonic_workspace_error(void* workspace, uint32_t* error_out, void* stream) {
  if (!error_out) return fail(SONIC_ERR_INVALID_ARGUMENT, "error_out must not be NULL");
  void* base = workspace;
  if (!base)
    if (sonic_status s = static_scratch(&base)) return s;
  cudaStream_t st = (cudaStream_t)stream;
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, base, sizeof(v), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && v) e = cudaMemsetAsync(base, 0, sizeof(v), st);
  if (e != cudaSuccess) return fail(SONIC_ERR_CUDA, std::string("sonic_workspace_error: ") + cudaGetErrorString(e));
  *error_out = v;
  return SONIC_OK;
}

extern "C" sonic_status sonic_fused_singular_static(const SonicSingularArgs* a, void* stream) {
  if (!a) return fail(SONIC_ERR_INVALID_ARGUMENT, "args must not be NULL");
  if (a->rows == 0) return SONIC_OK;
  // every argument check runs before the scratch is sized, carved or cleared
  if (sonic_status s = check_singular(a, true)) return s;
  if (!a->logits || a->logits_dtype != SONIC_DTYPE_BF16)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logits must be a non-NULL bf16 tensor");
  const size_t need = sonic_fused_singular_workspace_size(a);
  if (need > kStaticScratchBytes)
    return fail(SONIC_ERR_WORKSPACE, "sonic_fused_singular_static: this call needs " + std::to_string(need) +
                                         " bytes of scratch, more than the " + std::to_string(kStaticScratchBytes) +
                                         "-byte static scratch; use sonic_fused_singular with a workspace");
  void* base = nullptr;
  if (sonic_status s = static_scratch(&base)) return s;
  // the tickets start at zero (the candidate lists are written before use; the error word at
  // offset 0 is left set until sonic_workspace_error reads it)
  const Plan p = singular_plan(a->rows, a->vocab_size);
  const Workspace ws = carve(base, a->rows, a->rows, p.splits);
  const size_t off = (size_t)((char*)ws.tickets - (char*)base);
  if (off >= need) return fail(SONIC_ERR_UNSUPPORTED, "sonic_fused_singular_static: scratch layout");
  const cudaError_t e = cudaMemsetAsync(ws.tickets, 0, need - off, (cudaStream_t)stream);
  if (e != cudaSuccess) return fail(SONIC_ERR_CUDA, std::string("sonic_fused_singular_static: ") + cudaGetErrorString(e));
  SonicSingularArgs b = *a;
  b.workspace = base;
  b.workspace_bytes = kStaticScratchBytes;
  return sonic_fused_singular(&b, stream);
}
