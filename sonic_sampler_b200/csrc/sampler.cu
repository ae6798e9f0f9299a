// B200 (sm_100a) fused sampling / speculative-verification kernels behind the C ABI of
// include/sonic_b200.h.
//
// One launch per call. Each row (singular, top-k) or request (multistep) is cut into S
// column splits; one 256-thread CTA streams one split from HBM exactly once with 16-byte
// vector loads, applies the reference logit processors in registers, and keeps a
// shared-memory candidate buffer behind a rising value threshold, so most logits cost a
// load, a few bf16 ops and one compare. The split's exact top-128 (or, for greedy rows,
// its single best key) is written sorted to the workspace; the last CTA of the row or
// request to finish (per-row ticket in the workspace) merges the S sorted lists with warp
// bitonic merges and runs selection / verification. No second launch, no host sync.
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
#include <string>
#include <type_traits>

#include "../../include/sonic_b200.h"
#include "common.cuh"

namespace sonic {

constexpr int NT = 256;           // threads per CTA
constexpr int VPT = 8;            // consecutive columns per thread per chunk (16 B of bf16)
constexpr int CHUNK = NT * VPT;   // columns per CTA per chunk
constexpr int CAP = 4096;         // candidate buffer (keys) for single-row CTAs
constexpr int TARGET_CTAS = 592;  // 148 SMs x 4 resident CTAs
constexpr int MAX_SPLIT_COLS = 65536;
constexpr int MAX_SPLITS = 32;

struct Plan {
  int splits;
  int cols;
};

// Column split of a unit (row or request) of V columns; a pure function of the shapes so
// the workspace size never depends on the device.
static Plan split_plan(int64_t units, int64_t V) {
  int64_t s = units > 0 ? (TARGET_CTAS + units - 1) / units : 1;
  s = std::max<int64_t>(s, (V + MAX_SPLIT_COLS - 1) / MAX_SPLIT_COLS);
  s = std::min<int64_t>(s, MAX_SPLITS);
  s = std::max<int64_t>(s, 1);
  int64_t cols = (V + s - 1) / s;
  cols = (cols + CHUNK - 1) / CHUNK * CHUNK;
  cols = std::min<int64_t>(cols, MAX_SPLIT_COLS);
  Plan p;
  p.splits = (int)((V + cols - 1) / cols);
  p.cols = (int)cols;
  return p;
}

// workspace: [units][splits][128] u64 sorted candidate keys, then [units] u32 tickets.
static size_t workspace_bytes(int64_t units, int64_t V) {
  if (units <= 0) return 0;
  Plan p = split_plan(units, V);
  size_t cand = (size_t)units * p.splits * kMaxK * sizeof(uint64_t);
  size_t tick = (size_t)units * sizeof(uint32_t);
  return cand + ((tick + 255) / 256) * 256;
}

// ---------------------------------------------------------------------------------------
// small device utilities
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ int64_t load_index(const void* p, int32_t dtype, int64_t i) {
  return dtype == SONIC_DTYPE_I64 ? ((const int64_t*)p)[i] : (int64_t)((const int32_t*)p)[i];
}

__device__ __forceinline__ uint64_t ldcg64(const uint64_t* p) {
  return (uint64_t)__ldcg(reinterpret_cast<const unsigned long long*>(p));
}

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  return __ldcs(reinterpret_cast<const uint4*>(p));
}

struct RowParams {
  float rep, freq, pres, temp;
};

__device__ __forceinline__ RowParams load_row_params(const SonicSamplingParams& P, int64_t slot,
                                                     uint32_t ind) {
  RowParams rp;
  rp.rep = (P.repetition && (ind & 0x2)) ? bf2f(P.repetition[slot]) : 1.0f;
  rp.freq = (P.frequency && (ind & 0x4)) ? bf2f(P.frequency[slot]) : 0.0f;
  rp.pres = (P.presence && (ind & 0x8)) ? bf2f(P.presence[slot]) : 0.0f;
  rp.temp = (P.temperature && (ind & 0x20)) ? bf2f(P.temperature[slot]) : 1.0f;
  return rp;
}

// Which aux streams a row needs (reference ops/prologue.py:378-447).
struct Needs {
  bool proc, g, dec, ctx, bias, temp;
};

__device__ __forceinline__ Needs row_needs(const SonicSamplingParams& P, uint32_t ind) {
  Needs n;
  n.proc = (ind & 0x1F) != 0;
  n.g = n.proc && P.grammar && (ind & 0x1);
  n.dec = n.proc && P.decode_counts && (ind & 0xE);
  n.ctx = n.dec && P.context_counts && (ind & 0x2);
  n.bias = n.proc && P.bias && (ind & 0x10);
  n.temp = (ind & 0x20) != 0;
  return n;
}

// The reference logit processors for one logit (ops/prologue.py:29-114, 443-447), in its
// order and with its bf16 rounding after every operation.
__device__ __forceinline__ float apply_processors(float v, uint32_t ind, const Needs& n, bool gbit,
                                                  int32_t dec, int32_t ctx, float bias,
                                                  const RowParams& rp) {
  if (n.proc) {
    if (n.g && !gbit) v = __int_as_float(0xff800000);
    if (n.dec) {
      if (n.ctx) {
        const int32_t total = dec + ctx;
        const float s = total > 0 ? rp.rep : 1.0f;
        v = v < 0.0f ? rbf(__fmul_rn(v, s)) : rbf(__fdiv_rn(v, s));
      }
      if (ind & 0x4) v = rbf(__fsub_rn(v, rbf(__fmul_rn(rbf(__int2float_rn(dec)), rp.freq))));
      if (ind & 0x8) v = rbf(__fsub_rn(v, rbf(__fmul_rn(dec > 0 ? 1.0f : 0.0f, rp.pres))));
    }
    if (n.bias) v = rbf(__fadd_rn(v, bias));
  }
  if (n.temp) v = rbf(__fdiv_rn(v, rp.temp));
  return v;
}

// Greedy order key (ops/prologue.py:117-138 + ops/singular.py:71-131): value, then the
// lowest offset inside its block_n tile, then the lowest tile. -0.0 compares as +0.0.
__device__ __forceinline__ uint64_t greedy_key(float v, int64_t c, int log2bn) {
  uint32_t h = f2bf(v);
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
// per-thread chunk loading: 8 consecutive columns c..c+7 of one row
// ---------------------------------------------------------------------------------------

struct Aux8 {
  int32_t dec[VPT];
  int32_t ctx[VPT];
  float bias[VPT];
};

// aux-buffer columns of the 8 logits (shard offset, optional d2t remap)
struct Cols8 {
  int64_t col[VPT];
};

template <bool VEC>
__device__ __forceinline__ void load_logits8(const uint16_t* xrow, int64_t c, int nvalid,
                                             float (&x)[VPT]) {
  if (VEC && nvalid == VPT) {
    uint4 q = ld_stream(xrow + c);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(w[i] << 16);
      x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int j = 0; j < VPT; ++j) x[j] = j < nvalid ? bf2f(__ldcs(xrow + c + j)) : 0.0f;
  }
}

template <bool VEC>
__device__ __forceinline__ void load_logits8_f32(const float* xrow, int64_t c, int nvalid,
                                                 float (&x)[VPT]) {
  if (VEC && nvalid == VPT) {
    uint4 a = ld_stream(xrow + c), b = ld_stream(xrow + c + 4);
    x[0] = __uint_as_float(a.x); x[1] = __uint_as_float(a.y);
    x[2] = __uint_as_float(a.z); x[3] = __uint_as_float(a.w);
    x[4] = __uint_as_float(b.x); x[5] = __uint_as_float(b.y);
    x[6] = __uint_as_float(b.z); x[7] = __uint_as_float(b.w);
  } else {
#pragma unroll
    for (int j = 0; j < VPT; ++j) x[j] = j < nvalid ? __ldcs(xrow + c + j) : 0.0f;
  }
}

// VEC: the 8 aux columns are contiguous and 32-byte aligned (checked on the host).
template <bool VEC>
__device__ __forceinline__ void load_aux8(const SonicSamplingParams& P, const Needs& n, int64_t slot,
                                          const Cols8& cc, int nvalid, Aux8& a) {
  if (VEC && nvalid == VPT) {
    const int64_t c = cc.col[0];
    if (n.dec) {
      const int32_t* d = P.decode_counts + slot * P.counts_stride + c;
      uint4 p = ld_stream(d), q = ld_stream(d + 4);
      a.dec[0] = p.x; a.dec[1] = p.y; a.dec[2] = p.z; a.dec[3] = p.w;
      a.dec[4] = q.x; a.dec[5] = q.y; a.dec[6] = q.z; a.dec[7] = q.w;
    }
    if (n.ctx) {
      const int32_t* d = P.context_counts + slot * P.counts_stride + c;
      uint4 p = ld_stream(d), q = ld_stream(d + 4);
      a.ctx[0] = p.x; a.ctx[1] = p.y; a.ctx[2] = p.z; a.ctx[3] = p.w;
      a.ctx[4] = q.x; a.ctx[5] = q.y; a.ctx[6] = q.z; a.ctx[7] = q.w;
    }
    if (n.bias) {
      uint4 q = ld_stream(P.bias + slot * P.bias_stride + c);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a.bias[2 * i] = __uint_as_float(w[i] << 16);
        a.bias[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const bool ok = j < nvalid;
      const int64_t c = cc.col[j];
      a.dec[j] = (n.dec && ok) ? __ldcs(P.decode_counts + slot * P.counts_stride + c) : 0;
      a.ctx[j] = (n.ctx && ok) ? __ldcs(P.context_counts + slot * P.counts_stride + c) : 0;
      a.bias[j] = (n.bias && ok) ? bf2f(__ldcs(P.bias + slot * P.bias_stride + c)) : 0.0f;
    }
  }
}

template <bool VEC>
__device__ __forceinline__ uint32_t load_gbits8(const SonicSamplingParams& P, int64_t grow,
                                                const Cols8& cc, int nvalid) {
  const uint32_t* g = P.grammar + grow * P.grammar_stride;
  if (VEC && nvalid == VPT) {
    const int64_t c = cc.col[0];
    return (__ldg(g + (c >> 5)) >> (c & 31)) & 0xffu;
  }
  uint32_t bits = 0;
#pragma unroll
  for (int j = 0; j < VPT; ++j)
    if (j < nvalid) bits |= ((__ldg(g + (cc.col[j] >> 5)) >> (cc.col[j] & 31)) & 1u) << j;
  return bits;
}

// ---------------------------------------------------------------------------------------
// shared-memory candidate buffer
// ---------------------------------------------------------------------------------------

// Append the keys of the set bits of `m` (block-wide call, warp-aggregated atomics).
template <typename K>
__device__ __forceinline__ void cand_push(K* buf, int* cnt, const K (&key)[VPT], unsigned m,
                                          int lane) {
  const int np = __popc(m);
  int incl = np;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    int y = __shfl_up_sync(kFull, incl, d);
    if (lane >= d) incl += y;
  }
  const int total = __shfl_sync(kFull, incl, 31);
  if (total == 0) return;
  int base = 0;
  if (lane == 31) base = atomicAdd(cnt, total);
  base = __shfl_sync(kFull, base, 31);
  int pos = base + incl - np;
#pragma unroll
  for (int j = 0; j < VPT; ++j)
    if ((m >> j) & 1u) buf[pos++] = key[j];
}

template <typename K>
__device__ __forceinline__ float key_value(K k);
template <>
__device__ __forceinline__ float key_value<uint32_t>(uint32_t k) { return bf2f(dec16(k >> 16)); }
template <>
__device__ __forceinline__ float key_value<uint64_t>(uint64_t k) { return dec32((uint32_t)(k >> 32)); }

// Keep exactly the 128 largest keys of buf[0..*cnt) (requires *cnt > 128) and raise the
// value threshold to the 128th key's value. Block-wide; starts and ends synchronised.
template <typename K>
__device__ void cand_compact(K* buf, int* cnt, float* thr, K* top, int* tcnt, int* hist, int* bcast) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int n = *cnt;
  const K T = block_select<K, NT>(buf, n, kMaxK, hist, bcast);
  if (tid == 0) *tcnt = 0;
  __syncthreads();
  for (int base = 0; base < n; base += NT) {
    const int i = base + tid;
    const K k = i < n ? buf[i] : (K)0;
    const bool keep = i < n && k >= T;
    const unsigned b = __ballot_sync(kFull, keep);
    int off = 0;
    if (lane == 0 && b) off = atomicAdd(tcnt, __popc(b));
    off = __shfl_sync(kFull, off, 0);
    const int pos = off + __popc(b & ((1u << lane) - 1u));
    if (keep && pos < kMaxK) top[pos] = k;
  }
  __syncthreads();
  for (int i = tid; i < kMaxK; i += NT) buf[i] = top[i];
  if (tid == 0) {
    *cnt = kMaxK;
    *thr = key_value<K>(T);
  }
  __syncthreads();
}

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

template <typename K>
__device__ __forceinline__ K make_key(float v, int local);
template <>
__device__ __forceinline__ uint32_t make_key<uint32_t>(float v, int local) {
  return (enc16(f2bf(v)) << 16) | (uint32_t)(0xffff - local);
}
template <>
__device__ __forceinline__ uint64_t make_key<uint64_t>(float v, int local) {
  return ((uint64_t)enc32(v) << 32) | (uint64_t)(0xffffffffu - (uint32_t)local);
}

// Final per-split step: exact top-128 of the buffer, sorted, written as global keys.
template <typename K>
__device__ void split_finish(K* buf, int* cnt, float* thr, K* top, int* tcnt, int* hist, int* bcast,
                             int64_t c0, uint64_t* out) {
  __syncthreads();
  if (*cnt > kMaxK) cand_compact<K>(buf, cnt, thr, top, tcnt, hist, bcast);
  const int n = *cnt;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    uint64_t k[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * lane + j;
      k[j] = i < n ? to_global<K>(buf[i], c0) : 0ull;
    }
    warp_sort128_desc(k, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) __stcg(reinterpret_cast<unsigned long long*>(out + 4 * lane + j), (unsigned long long)k[j]);
    __threadfence();
  }
}

// Ticket: true in the last CTA of the unit to arrive; that CTA also re-arms the ticket.
__device__ __forceinline__ bool arrive_last(uint32_t* ticket, int splits, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(ticket, 1u);
    const bool last = prev == (uint32_t)(splits - 1);
    if (last) *ticket = 0;
    *flag = last;
  }
  __syncthreads();
  const bool last = *flag != 0;
  if (last) __threadfence();
  return last;
}

// Fold `splits` sorted candidate lists (u64 keys, descending) into one (warp-wide).
__device__ __forceinline__ void warp_fold_lists(const uint64_t* lists, int splits, int lane,
                                                uint64_t (&acc)[4]) {
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

// cumulative_masking (ops/base.py:95-129) on the sorted top-128 held 4 per lane.
__device__ __forceinline__ void warp_masking(const SonicSamplingParams& P, int64_t slot, uint32_t ind,
                                             float (&v)[4], float maximum, int lane) {
  const float ninf = __int_as_float(0xff800000);
  if ((ind & 0x80) && P.top_k) {
    const int32_t k = P.top_k[slot];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(4 * lane + j < k)) v[j] = ninf;
  }
  if ((ind & 0x100) && P.top_p) {
    float e[4], lad[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) e[j] = dexp(__fsub_rn(v[j], maximum));
    warp_ladder128(e, lad, lane);
    const float total = __shfl_sync(kFull, lad[3], 31);
    const float scale = __fmul_rn(total, bf2f(P.top_p[slot]));
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(lad[j] <= scale || (lane == 0 && j == 0))) v[j] = ninf;
  }
  if ((ind & 0x200) && P.min_p) {
    const float pivot = __fadd_rn(dlog(bf2f(P.min_p[slot])), maximum);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (!(v[j] >= pivot)) v[j] = ninf;
  }
}

// log_softmax (ops/base.py:66-72) of 128 values held 4 per lane.
__device__ __forceinline__ void warp_log_softmax(const float (&v)[4], float maximum, float (&ls)[4]) {
  float sc[4], e[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sc[j] = __fsub_rn(v[j], maximum);
    e[j] = dexp(sc[j]);
  }
  const float lse = dlog(warp_sum128(e));
#pragma unroll
  for (int j = 0; j < 4; ++j) ls[j] = __fsub_rn(sc[j], lse);
}

__device__ __forceinline__ void store_float(void* base, int32_t dtype, int64_t i, float x) {
  if (dtype == SONIC_DTYPE_F32)
    ((float*)base)[i] = x;
  else
    ((uint16_t*)base)[i] = f2bf(x);
}

__device__ __forceinline__ int64_t load_slot(const SonicSamplingParams& P, int64_t unit) {
  return P.slot_mapping ? load_index(P.slot_mapping, P.slot_dtype, unit) : unit;
}

// ---------------------------------------------------------------------------------------
// shared memory of a single-row CTA
// ---------------------------------------------------------------------------------------

template <typename K>
struct RowSmem {
  K buf[CAP];
  K top[kMaxK];
  int hist[256];
  int bcast[4];
  int cnt;
  int tcnt;
  int flag;
  float thr;
  uint64_t warp_best[NT / 32];
  int32_t toks[SONIC_MAX_LOOKAHEAD + 1];
};

// ---------------------------------------------------------------------------------------
// fused singular: prologue + top-128 per split + merge + selection
// (ops/prologue.py:272 + ops/singular.py:154)
// ---------------------------------------------------------------------------------------

template <bool VEC, bool INDIRECT>
__global__ void __launch_bounds__(NT) singular_kernel(const SonicSingularArgs a, int splits, int cols,
                                                      int log2bn, uint64_t* cand, uint32_t* tickets) {
  __shared__ RowSmem<uint32_t> sm;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int64_t r = blockIdx.y;
  const SonicSamplingParams& P = a.params;
  const int64_t c0 = (int64_t)split * cols;
  const int64_t c1 = min((int64_t)a.vocab_size, c0 + cols);

  pdl_wait();

  const int64_t slot = load_slot(P, r);
  if (slot < 0 || (P.num_slots > 0 && slot >= P.num_slots)) {
    // out-of-range slot id: no CTA of this row touches per-slot buffers or the ticket
    if (split == 0 && tid == 0) a.tokens[r * a.tokens_stride] = -1;
    return;
  }
  const uint32_t ind = P.indicators[slot];
  const Needs nd = row_needs(P, ind);
  const RowParams rp = load_row_params(P, slot, ind);
  const bool greedy = (ind & 0x40) != 0;
  const int ntok = (a.drafted_tokens && nd.dec) ? a.lookahead : 0;
  if (tid < ntok) sm.toks[tid] = a.drafted_tokens[slot * a.drafted_stride + tid];
  if (tid == 0) {
    sm.cnt = 0;
    sm.thr = __int_as_float(0xff800000);
  }
  __syncthreads();

  const uint16_t* xrow = (const uint16_t*)a.logits + r * a.logits_stride;
  uint64_t best = 0;

#pragma unroll 1
  for (int64_t cb = c0; cb < c1; cb += CHUNK) {
    const int64_t c = cb + (int64_t)VPT * tid;
    const int nvalid = (int)max((int64_t)0, min((int64_t)VPT, c1 - c));
    float x[VPT];
    load_logits8<VEC>(xrow, c, nvalid, x);
    if (nd.proc || nd.temp) {
      Cols8 cc;
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        int64_t col = c + j + a.shard_offset;
        if (INDIRECT && nd.proc && j < nvalid) col = load_index(a.d2t, a.d2t_dtype, col);
        cc.col[j] = col;
      }
      Aux8 ax;
      load_aux8<VEC && !INDIRECT>(P, nd, slot, cc, nvalid, ax);
      const uint32_t gb = nd.g ? load_gbits8<VEC && !INDIRECT>(P, slot, cc, nvalid) : 0xffu;
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        int32_t dec = ax.dec[j];
        for (int s = 0; s < ntok; ++s) dec += (sm.toks[s] == cc.col[j]);
        x[j] = apply_processors(x[j], ind, nd, (gb >> j) & 1u, dec, ax.ctx[j], ax.bias[j], rp);
      }
    }
    if (greedy) {
#pragma unroll
      for (int j = 0; j < VPT; ++j)
        if (j < nvalid) best = umax(best, greedy_key(x[j], c + j, log2bn));
    } else {
      const float thr = sm.thr;
      uint32_t key[VPT];
      unsigned m = 0;
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        key[j] = make_key<uint32_t>(x[j], (int)(c + j - c0));
        if (j < nvalid && x[j] >= thr) m |= 1u << j;
      }
      cand_push<uint32_t>(sm.buf, &sm.cnt, key, m, lane);
      __syncthreads();
      const bool full = sm.cnt > CAP - CHUNK;
      __syncthreads();
      if (full) cand_compact<uint32_t>(sm.buf, &sm.cnt, &sm.thr, sm.top, &sm.tcnt, sm.hist, sm.bcast);
    }
  }
  pdl_trigger();

  uint64_t* lists = cand + (uint64_t)r * splits * kMaxK;
  if (greedy) {
    best = warp_max_u64(best);
    if (lane == 0) sm.warp_best[warp] = best;
    __syncthreads();
    if (tid == 0) {
      uint64_t b = sm.warp_best[0];
      for (int w = 1; w < NT / 32; ++w) b = umax(b, sm.warp_best[w]);
      __stcg(reinterpret_cast<unsigned long long*>(lists + (int64_t)split * kMaxK), (unsigned long long)b);
      __threadfence();
    }
  } else {
    split_finish<uint32_t>(sm.buf, &sm.cnt, &sm.thr, sm.top, &sm.tcnt, sm.hist, sm.bcast, c0,
                           lists + (int64_t)split * kMaxK);
  }

  if (!arrive_last(tickets + r, splits, &sm.flag)) return;
  if (warp != 0) return;

  // ---- merge + selection (one warp) ----
  const uint32_t flags = a.flags;
  if (greedy) {
    uint64_t b = 0;
    for (int s = lane; s < splits; s += 32) b = umax(b, ldcg64(lists + (int64_t)s * kMaxK));
    b = warp_max_u64(b);
    int64_t token = greedy_col(b, log2bn);
    if (a.d2t) token = load_index(a.d2t, a.d2t_dtype, token);
    if (lane == 0) {
      if ((flags & SONIC_FLAG_UPDATE_COUNTS) && token >= 0 && token < P.counts_stride) {
        int32_t* d = P.decode_counts + slot * P.counts_stride + token;
        *d = (flags & SONIC_FLAG_PREFILL) ? 1 : *d + 1;
      }
      a.tokens[r * a.tokens_stride] = (int32_t)token;
    }
    return;
  }

  uint64_t k[4];
  warp_fold_lists(lists, splits, lane, k);
  float v[4];
  int64_t idx[4];
  decode_keys(k, v, idx);
  const float vmax = __shfl_sync(kFull, v[0], 0);
  if (ind & 0x380) warp_masking(P, slot, ind, v, vmax, lane);
  int64_t tok[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) tok[j] = a.d2t ? load_index(a.d2t, a.d2t_dtype, idx[j]) : idx[j];
  float diff[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (flags & SONIC_FLAG_PHILOX)
      diff[j] = __fsub_rn(v[j], philox_log_exponential(a.philox_seed, a.philox_offset, (uint32_t)slot,
                                                        (uint32_t)tok[j]));
    else
      diff[j] = (a.target_vocab > 0 && (tok[j] < 0 || tok[j] >= a.target_vocab))
                    ? __int_as_float(0xff800000)
                    : rbf(__fsub_rn(v[j], bf2f(a.gumbel[slot * a.gumbel_stride + tok[j]])));
  }
  const int sel = warp_argmax128(diff, lane);
  const int64_t token = warp_pick128(tok, sel);
  if (lane == 0 && (flags & SONIC_FLAG_UPDATE_COUNTS) && token >= 0 && token < P.counts_stride) {
    int32_t* d = P.decode_counts + slot * P.counts_stride + token;
    *d = (flags & SONIC_FLAG_PREFILL) ? 1 : *d + 1;
  }
  if (flags & (SONIC_FLAG_LOGPROBS | SONIC_FLAG_PROBABILITIES)) {
    float ls[4];
    warp_log_softmax(v, __shfl_sync(kFull, v[0], 0), ls);
    if ((flags & SONIC_FLAG_LOGPROBS) && a.logprobs) {
      const float lsel = warp_pick128(ls, sel);
      if (lane == 0) store_float(a.logprobs, a.logprobs_dtype, r * a.logprobs_stride, lsel);
      if (a.max_top_logprobs > 0 && (ind & 0x400) && a.top_logprob_values && P.top_logprobs) {
        const int z = min(P.top_logprobs[slot], a.max_top_logprobs);
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
        if (a.target_vocab <= 0 || (tok[j] >= 0 && tok[j] < a.target_vocab))
          store_float(a.probabilities, a.probabilities_dtype, slot * a.probabilities_stride + tok[j], p);
      }
    }
  }
  if (lane == 0) a.tokens[r * a.tokens_stride] = (int32_t)token;
}

// ---------------------------------------------------------------------------------------
// bounded top-k (ops/topk/bitpack.py:99 + ops/topk/unpack.py:312)
// ---------------------------------------------------------------------------------------

template <bool VEC, bool F32>
__global__ void __launch_bounds__(NT) topk_kernel(const SonicTopKArgs a, int splits, int cols,
                                                  uint64_t* cand, uint32_t* tickets) {
  using K = typename std::conditional<F32, uint64_t, uint32_t>::type;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  RowSmem<K>& sm = *reinterpret_cast<RowSmem<K>*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int64_t r = blockIdx.y;
  const int64_t c0 = (int64_t)split * cols;
  const int64_t c1 = min((int64_t)a.vocab_size, c0 + cols);

  pdl_wait();
  if (tid == 0) {
    sm.cnt = 0;
    sm.thr = __int_as_float(0xff800000);
  }
  __syncthreads();

#pragma unroll 1
  for (int64_t cb = c0; cb < c1; cb += CHUNK) {
    const int64_t c = cb + (int64_t)VPT * tid;
    const int nvalid = (int)max((int64_t)0, min((int64_t)VPT, c1 - c));
    float x[VPT];
    if (F32)
      load_logits8_f32<VEC>((const float*)a.logits + r * a.logits_stride, c, nvalid, x);
    else
      load_logits8<VEC>((const uint16_t*)a.logits + r * a.logits_stride, c, nvalid, x);
    const float thr = sm.thr;
    K key[VPT];
    unsigned m = 0;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      key[j] = make_key<K>(x[j], (int)(c + j - c0));
      if (j < nvalid && x[j] >= thr) m |= 1u << j;
    }
    cand_push<K>(sm.buf, &sm.cnt, key, m, lane);
    __syncthreads();
    const bool full = sm.cnt > CAP - CHUNK;
    __syncthreads();
    if (full) cand_compact<K>(sm.buf, &sm.cnt, &sm.thr, sm.top, &sm.tcnt, sm.hist, sm.bcast);
  }
  pdl_trigger();

  uint64_t* lists = cand + (uint64_t)r * splits * kMaxK;
  split_finish<K>(sm.buf, &sm.cnt, &sm.thr, sm.top, &sm.tcnt, sm.hist, sm.bcast, c0,
                  lists + (int64_t)split * kMaxK);
  if (!arrive_last(tickets + r, splits, &sm.flag)) return;
  if (warp != 0) return;

  uint64_t k[4];
  warp_fold_lists(lists, splits, lane, k);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = 4 * lane + j;
    if (i >= a.k) continue;
    const uint32_t e = (uint32_t)(k[j] >> 32);
    const int64_t col = (int64_t)(0xffffffffu - (uint32_t)k[j]);
    const int64_t o = r * a.k + i;
    const float val = F32 ? dec32(e) : bf2f(dec16(e));
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
// fused multistep: prologue over all gamma+1 rows of a request (aux rows read once),
// merge per row, softmax of the masked candidates, chain verification
// (ops/prologue.py:272 + ops/multistep.py:76 + ops/verify.py:244)
// ---------------------------------------------------------------------------------------

constexpr int MS_MAX_STEPS = SONIC_MAX_LOOKAHEAD + 1;
constexpr int MS_GROUP = 8;  // logits rows loaded together per chunk

struct MsSmem {
  int hist[256];
  int bcast[4];
  int cnt[MS_MAX_STEPS];
  float thr[MS_MAX_STEPS];
  int tcnt;
  int flag;
  int32_t drafted[MS_MAX_STEPS];
  unsigned long long best[MS_MAX_STEPS];
  uint32_t top[kMaxK];
  // after the streaming phase (last CTA only):
  float prob[MS_MAX_STEPS][kMaxK];
  int32_t cand[MS_MAX_STEPS][kMaxK];
  int64_t gsel[MS_MAX_STEPS];
};

static int ms_cap(int steps) { return steps <= 8 ? 3072 : 2176; }

static size_t ms_smem_bytes(int steps) {
  return sizeof(MsSmem) + (size_t)steps * ms_cap(steps) * sizeof(uint32_t);
}

template <bool VEC>
__global__ void __launch_bounds__(NT) multistep_kernel(const SonicMultistepArgs a, int splits, int cols,
                                                       int log2bn, int cap, uint64_t* cand,
                                                       uint32_t* tickets) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  MsSmem& sm = *reinterpret_cast<MsSmem*>(smem_raw);
  uint32_t* bufs = reinterpret_cast<uint32_t*>(smem_raw + sizeof(MsSmem));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x;
  const int64_t b = blockIdx.y;
  const SonicSamplingParams& P = a.params;
  const int G = a.lookahead;
  const int64_t c0 = (int64_t)split * cols;
  const int64_t c1 = min((int64_t)a.vocab_size, c0 + cols);

  pdl_wait();

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
    if (split == 0 && tid == 0) a.offsets[b] = -1;
    return;
  }
  const uint32_t ind = P.indicators[slot];
  const Needs nd = row_needs(P, ind);
  const RowParams rp = load_row_params(P, slot, ind);
  const bool greedy = (ind & 0x40) != 0;
  if (tid < T) {
    sm.drafted[tid] = a.drafted_tokens[margin + tid];
    sm.cnt[tid] = 0;
    sm.thr[tid] = __int_as_float(0xff800000);
    sm.best[tid] = 0ull;
  }
  __syncthreads();

#pragma unroll 1
  for (int64_t cb = c0; cb < c1; cb += CHUNK) {
    const int64_t c = cb + (int64_t)VPT * tid;
    const int nvalid = (int)max((int64_t)0, min((int64_t)VPT, c1 - c));
    Cols8 cc;
#pragma unroll
    for (int j = 0; j < VPT; ++j) cc.col[j] = c + j + a.shard_offset;
    Aux8 ax;
    if (nd.proc) load_aux8<VEC>(P, nd, slot, cc, nvalid, ax);
#pragma unroll 1
    for (int s0 = 0; s0 < T; s0 += MS_GROUP) {
      // issue the logits loads of up to MS_GROUP rows before touching any of them
      float xs[MS_GROUP][VPT];
#pragma unroll
      for (int g = 0; g < MS_GROUP; ++g)
        if (s0 + g < T)
          load_logits8<VEC>((const uint16_t*)a.logits + (margin + s0 + g) * a.logits_stride, c, nvalid, xs[g]);
#pragma unroll
      for (int g = 0; g < MS_GROUP; ++g) {
        const int s = s0 + g;
        if (s >= T) break;
        float (&x)[VPT] = xs[g];
        if (nd.proc || nd.temp) {
          const uint32_t gb = nd.g ? load_gbits8<VEC>(P, slot * (G + 1) + s, cc, nvalid) : 0xffu;
#pragma unroll
          for (int j = 0; j < VPT; ++j) {
            int32_t dec = nd.proc ? ax.dec[j] : 0;
            if (nd.dec)
              for (int q = 0; q < s; ++q) dec += (sm.drafted[q] == cc.col[j]);
            x[j] = apply_processors(x[j], ind, nd, (gb >> j) & 1u, dec, nd.proc ? ax.ctx[j] : 0,
                                    nd.proc ? ax.bias[j] : 0.0f, rp);
          }
        }
        if (greedy) {
          uint64_t best = 0;
#pragma unroll
          for (int j = 0; j < VPT; ++j)
            if (j < nvalid) best = umax(best, greedy_key(x[j], c + j, log2bn));
          best = warp_max_u64(best);
          if (lane == 0 && best) atomicMax(&sm.best[s], (unsigned long long)best);
        } else {
          const float thr = sm.thr[s];
          uint32_t key[VPT];
          unsigned m = 0;
#pragma unroll
          for (int j = 0; j < VPT; ++j) {
            key[j] = make_key<uint32_t>(x[j], (int)(c + j - c0));
            if (j < nvalid && x[j] >= thr) m |= 1u << j;
          }
          cand_push<uint32_t>(bufs + (int64_t)s * cap, &sm.cnt[s], key, m, lane);
        }
      }
    }
    if (!greedy) {
      __syncthreads();
      unsigned full = 0;
      for (int s = 0; s < T; ++s)
        if (sm.cnt[s] > cap - CHUNK) full |= 1u << s;
      __syncthreads();
#pragma unroll 1
      for (int s = 0; s < T; ++s)
        if ((full >> s) & 1u)
          cand_compact<uint32_t>(bufs + (int64_t)s * cap, &sm.cnt[s], &sm.thr[s], sm.top, &sm.tcnt,
                                 sm.hist, sm.bcast);
    }
  }
  pdl_trigger();

  // per-row candidate lists: row (margin + s), split
  const int64_t L = a.total_rows;
  (void)L;
  if (greedy) {
    __syncthreads();
    if (tid < T) {
      __stcg(reinterpret_cast<unsigned long long*>(cand + ((margin + tid) * splits + split) * kMaxK), sm.best[tid]);
      __threadfence();
    }
  } else {
#pragma unroll 1
    for (int s = 0; s < T; ++s)
      split_finish<uint32_t>(bufs + (int64_t)s * cap, &sm.cnt[s], &sm.thr[s], sm.top, &sm.tcnt, sm.hist,
                             sm.bcast, c0, cand + ((margin + s) * splits + split) * kMaxK);
  }
  if (!arrive_last(tickets + b, splits, &sm.flag)) return;

  // ---- per-row merge (warp w handles rows w, w+8, ...) ----
  const float ninf = __int_as_float(0xff800000);
  for (int s = warp; s < T; s += NT / 32) {
    const uint64_t* lists = cand + (margin + s) * splits * kMaxK;
    if (greedy) {
      uint64_t bk = 0;
      for (int q = lane; q < splits; q += 32) bk = umax(bk, ldcg64(lists + (int64_t)q * kMaxK));
      bk = warp_max_u64(bk);
      const int64_t g = greedy_col(bk, log2bn);
      if (lane == 0) {
        sm.gsel[s] = g;
        if (a.indices) a.indices[margin * kMaxK + s] = (int32_t)g;
      }
    } else {
      uint64_t k[4];
      warp_fold_lists(lists, splits, lane, k);
      float v[4];
      int64_t idx[4];
      decode_keys(k, v, idx);
      const float vmax = __shfl_sync(kFull, v[0], 0);
      if (ind & 0x380) warp_masking(P, slot, ind, v, vmax, lane);
      float ls[4];
      warp_log_softmax(v, vmax, ls);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = 4 * lane + j;
        const float p = dexp(ls[j]);
        sm.prob[s][i] = p;
        sm.cand[s][i] = (int32_t)idx[j];
        if (a.values) a.values[(margin + s) * kMaxK + i] = p;
        if (a.indices) a.indices[(margin + s) * kMaxK + i] = (int32_t)idx[j];
      }
    }
  }
  __syncthreads();
  if (warp != 0) return;
  (void)ninf;

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
      float u = bf2f(a.uniform[slot * a.uniform_stride + accepted]);
      if (stochastic_draft && dr[accepted] >= 0 && dr[accepted] < a.vocab_size) {
        const int64_t qi = slot * a.draft_stride + accepted * a.draft_step_stride + dr[accepted];
        if (a.draft_dtype == SONIC_DTYPE_F32)
          u = __fmul_rn(u, ((const float*)a.draft_probs)[qi]);
        else
          u = rbf(__fmul_rn(u, bf2f(((const uint16_t*)a.draft_probs)[qi])));
      }
      bool keep = false;
#pragma unroll
      for (int s = 0; s < MS_MAX_STEPS; ++s)
        if (s == accepted) keep = u <= targets[s];
      if (!keep) break;
    }
    // rejection_sample (verify.py:157-241)
    float score[4];
    int32_t pos[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = 4 * lane + j;
      const float sc = sm.prob[accepted][i];
      pos[j] = sm.cand[accepted][i];
      float rr;
      if (accepted == T - 1)
        rr = sc;
      else if (!stochastic_draft)
        rr = (pos[j] == sm.drafted[accepted]) ? 0.0f : sc;
      else {
        const int64_t qi = slot * a.draft_stride + accepted * a.draft_step_stride + pos[j];
        const float q = a.draft_dtype == SONIC_DTYPE_F32 ? ((const float*)a.draft_probs)[qi]
                                                         : bf2f(((const uint16_t*)a.draft_probs)[qi]);
        rr = __fsub_rn(sc, q);
        rr = rr < 0.0f ? 0.0f : (rr > 1.0f ? 1.0f : rr);
      }
      const float g = bf2f(a.gumbel[slot * a.gumbel_stride + accepted * a.gumbel_step_stride + pos[j]]);
      score[j] = __fsub_rn(dlog(rr), g);
    }
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
          const int z = min(P.top_logprobs[slot], a.max_top_logprobs);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int i = 4 * lane + j;
            if (i < z) {
              store_float(a.top_logprob_values, a.logprobs_dtype, (margin + s) * a.top_stride + i, dlog(sm.prob[s][i]));
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

// Vector (16-byte) aux loads need every row start and column offset 32-byte aligned.
static bool params_vec_ok(const SonicSamplingParams& P, int64_t shard_offset) {
  bool ok = (shard_offset % 32) == 0;
  if (P.decode_counts) ok = ok && aligned(P.decode_counts, 16) && (P.counts_stride % 4) == 0;
  if (P.context_counts) ok = ok && aligned(P.context_counts, 16) && (P.counts_stride % 4) == 0;
  if (P.bias) ok = ok && aligned(P.bias, 16) && (P.bias_stride % 8) == 0;
  return ok;
}

static sonic_status check_params(const SonicSamplingParams& P) {
  if (!P.indicators) return fail(SONIC_ERR_INVALID_ARGUMENT, "indicators must not be NULL");
  if (P.slot_mapping && P.slot_dtype != SONIC_DTYPE_I32 && P.slot_dtype != SONIC_DTYPE_I64)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "slot_mapping dtype must be i32 or i64");
  return SONIC_OK;
}

}  // namespace sonic

using namespace sonic;

extern "C" {

int32_t sonic_abi_version(void) { return SONIC_B200_ABI_VERSION; }

const char* sonic_last_error(void) { return g_last_error.c_str(); }

size_t sonic_fused_singular_workspace_size(const SonicSingularArgs* a) {
  return a ? workspace_bytes(a->rows, a->vocab_size) : 0;
}

size_t sonic_fused_multistep_workspace_size(const SonicMultistepArgs* a) {
  if (!a) return 0;
  // candidate lists per row, tickets per request
  if (a->batch_size <= 0) return 0;
  Plan p = split_plan(a->batch_size, a->vocab_size);
  int64_t rows = a->total_rows > 0 ? a->total_rows : (int64_t)a->batch_size * (a->lookahead + 1);
  size_t cand = (size_t)rows * p.splits * kMaxK * sizeof(uint64_t);
  size_t tick = (size_t)a->batch_size * sizeof(uint32_t);
  return cand + ((tick + 255) / 256) * 256;
}

size_t sonic_bounded_topk_workspace_size(const SonicTopKArgs* a) {
  return a ? workspace_bytes(a->rows, a->vocab_size) : 0;
}

sonic_status sonic_fused_singular(const SonicSingularArgs* a, void* stream) {
  if (!a) return fail(SONIC_ERR_INVALID_ARGUMENT, "args must not be NULL");
  if (a->rows == 0) return SONIC_OK;
  if (a->rows < 0 || a->rows > 65535) return fail(SONIC_ERR_INVALID_ARGUMENT, "rows must be in [0, 65535]");
  if (a->vocab_size < kMaxK) return fail(SONIC_ERR_INVALID_ARGUMENT, "vocab_size must be >= 128");
  if (sonic_status s = check_block_n(a->block_n)) return s;
  if (sonic_status s = check_params(a->params)) return s;
  if (!a->logits || a->logits_dtype != SONIC_DTYPE_BF16)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logits must be a non-NULL bf16 tensor");
  if (!a->tokens) return fail(SONIC_ERR_INVALID_ARGUMENT, "tokens must not be NULL");
  if (a->lookahead < 0 || a->lookahead > SONIC_MAX_LOOKAHEAD)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "lookahead must be in [0, 15]");
  if (a->d2t && a->d2t_dtype != SONIC_DTYPE_I32 && a->d2t_dtype != SONIC_DTYPE_I64)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "d2t dtype must be i32 or i64");
  if (!(a->flags & SONIC_FLAG_PHILOX) && !a->gumbel)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "gumbel noise must not be NULL without SONIC_FLAG_PHILOX");
  if ((a->flags & SONIC_FLAG_UPDATE_COUNTS) && !a->params.decode_counts)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "`update_counts` is True but `decode_counts` is None");
  if ((a->flags & SONIC_FLAG_PROBABILITIES) && a->probabilities &&
      a->probabilities_dtype != SONIC_DTYPE_BF16 && a->probabilities_dtype != SONIC_DTYPE_F32)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "probabilities dtype must be bf16 or f32");
  if (a->max_top_logprobs < 0 || a->max_top_logprobs > kMaxK)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "max_top_logprobs must be in [0, 128]");
  if (a->logprobs_dtype != SONIC_DTYPE_BF16 && a->logprobs_dtype != SONIC_DTYPE_F32)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logprobs dtype must be bf16 or f32");
  const size_t need = workspace_bytes(a->rows, a->vocab_size);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(SONIC_ERR_WORKSPACE, "workspace smaller than sonic_fused_singular_workspace_size()");
  Plan p = split_plan(a->rows, a->vocab_size);
  uint64_t* cand = (uint64_t*)a->workspace;
  uint32_t* tick = (uint32_t*)((char*)a->workspace + (size_t)a->rows * p.splits * kMaxK * sizeof(uint64_t));
  const bool vec = aligned(a->logits, 16) && (a->logits_stride % 8) == 0 && params_vec_ok(a->params, a->shard_offset);
  const bool ind = a->d2t != nullptr;
  dim3 grid(p.splits, a->rows);
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = (a->flags & SONIC_FLAG_PDL) != 0;
  const int l2 = ilog2(a->block_n);
  cudaError_t e;
  if (ind)
    e = vec ? launch(singular_kernel<true, true>, grid, 0, st, pdl, *a, p.splits, p.cols, l2, cand, tick)
            : launch(singular_kernel<false, true>, grid, 0, st, pdl, *a, p.splits, p.cols, l2, cand, tick);
  else
    e = vec ? launch(singular_kernel<true, false>, grid, 0, st, pdl, *a, p.splits, p.cols, l2, cand, tick)
            : launch(singular_kernel<false, false>, grid, 0, st, pdl, *a, p.splits, p.cols, l2, cand, tick);
  return check_launch(e, "sonic_fused_singular");
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
  const size_t need = workspace_bytes(a->rows, a->vocab_size);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(SONIC_ERR_WORKSPACE, "workspace smaller than sonic_bounded_topk_workspace_size()");
  Plan p = split_plan(a->rows, a->vocab_size);
  uint64_t* cand = (uint64_t*)a->workspace;
  uint32_t* tick = (uint32_t*)((char*)a->workspace + (size_t)a->rows * p.splits * kMaxK * sizeof(uint64_t));
  const bool f32 = a->logits_dtype == SONIC_DTYPE_F32;
  const bool vec = aligned(a->logits, 16) && (a->logits_stride % (f32 ? 4 : 8)) == 0;
  dim3 grid(p.splits, a->rows);
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = (a->flags & SONIC_FLAG_PDL) != 0;
  cudaError_t e;
  if (f32) {
    const size_t smem = sizeof(RowSmem<uint64_t>);
    auto k = vec ? topk_kernel<true, true> : topk_kernel<false, true>;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) e = launch(k, grid, smem, st, pdl, *a, p.splits, p.cols, cand, tick);
  } else {
    const size_t smem = sizeof(RowSmem<uint32_t>);
    auto k = vec ? topk_kernel<true, false> : topk_kernel<false, false>;
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) e = launch(k, grid, smem, st, pdl, *a, p.splits, p.cols, cand, tick);
  }
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
  if (!a->gumbel || !a->uniform)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "gumbel and uniform noise must not be NULL");
  if (a->draft_probs && a->draft_dtype != SONIC_DTYPE_F32 && a->draft_dtype != SONIC_DTYPE_BF16)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "draft probabilities dtype must be f32 or bf16");
  if ((a->flags & SONIC_FLAG_UPDATE_COUNTS) && !a->params.decode_counts)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "`update_counts` is True but `decode_counts` is None");
  if (a->max_top_logprobs < 0 || a->max_top_logprobs > kMaxK)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "max_top_logprobs must be in [0, 128]");
  if (a->logprobs_dtype != SONIC_DTYPE_BF16 && a->logprobs_dtype != SONIC_DTYPE_F32)
    return fail(SONIC_ERR_INVALID_ARGUMENT, "logprobs dtype must be bf16 or f32");
  const size_t need = sonic_fused_multistep_workspace_size(a);
  if (!a->workspace || a->workspace_bytes < need)
    return fail(SONIC_ERR_WORKSPACE, "workspace smaller than sonic_fused_multistep_workspace_size()");
  Plan p = split_plan(a->batch_size, a->vocab_size);
  const int64_t rows = a->total_rows > 0 ? a->total_rows : (int64_t)a->batch_size * (a->lookahead + 1);
  uint64_t* cand = (uint64_t*)a->workspace;
  uint32_t* tick = (uint32_t*)((char*)a->workspace + (size_t)rows * p.splits * kMaxK * sizeof(uint64_t));
  const bool vec = aligned(a->logits, 16) && (a->logits_stride % 8) == 0 && params_vec_ok(a->params, a->shard_offset);
  const int steps = a->lookahead + 1;
  const int cap = ms_cap(steps);
  const size_t smem = ms_smem_bytes(steps);
  dim3 grid(p.splits, a->batch_size);
  cudaStream_t st = (cudaStream_t)stream;
  const bool pdl = (a->flags & SONIC_FLAG_PDL) != 0;
  auto k = vec ? multistep_kernel<true> : multistep_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) e = launch(k, grid, smem, st, pdl, *a, p.splits, p.cols, ilog2(a->block_n), cap, cand, tick);
  return check_launch(e, "sonic_fused_multistep");
}

}  // extern "C"
