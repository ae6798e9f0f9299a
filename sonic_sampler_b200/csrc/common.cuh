// Shared device helpers for the B200 sampler kernels: bf16 arithmetic, order-preserving key
// encodings, deterministic exp/log, Philox noise, and warp/block selection primitives.
//
// Numerics contract. Every bf16 operation of the reference prologue (ops/prologue.py) is done
// as an fp32 operation followed by round-to-nearest-even to bf16; for these operands that is
// exactly the bf16 result (fp32 products of two bf16 values are exact; sums and quotients of
// bf16 values never fall within 2 fp32 ulps of a bf16 rounding midpoint). This file is
// compiled with --fmad=false so no multiply-add is contracted behind the code's back; the
// fused multiply-adds below are explicit.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace sonic {

constexpr int kMaxK = 128;
constexpr unsigned kFull = 0xffffffffu;

// ---------------------------------------------------------------------------------------
// bf16 helpers (reference ops/encoding.py:31-123)
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ float bf2f(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// round an fp32 value to the nearest bf16 (ties to even) and widen back.
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }

// encode_block: bf16 bits -> u16 whose unsigned order is the value order (-0 < +0).
__device__ __forceinline__ uint32_t enc16(uint32_t h) {
  return (h & 0x8000u) ? (h ^ 0xffffu) : (h ^ 0x8000u);
}

__device__ __forceinline__ uint32_t dec16(uint32_t e) {
  return (e & 0x8000u) ? (e ^ 0x8000u) : (e ^ 0xffffu);
}

__device__ __forceinline__ uint32_t enc32(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float dec32(uint32_t e) {
  return __uint_as_float((e & 0x80000000u) ? (e & 0x7fffffffu) : ~e);
}

// ---------------------------------------------------------------------------------------
// exp / log: Cody-Waite reduction with a degree-7 Taylor polynomial for exp, and the atanh
// series for log. Bit-identical to the host restatement used by the tests.
// ---------------------------------------------------------------------------------------

constexpr float kLog2e = 1.44269502162933349609375f;   // 0x3fb8aa3b
constexpr float kLn2Hi = 0.693145751953125f;           // 0x3f317200 (16 significant bits)
constexpr float kLn2Lo = 1.428606765330187e-06f;       // 0x35bfbe8e = ln2 - kLn2Hi
constexpr float kSqrt2 = 1.41421353816986083984375f;   // 0x3fb504f3

__device__ __forceinline__ float dexp(float x) {
  if (x != x) return x;
  if (x > 88.7228317f) return __int_as_float(0x7f800000);
  if (x < -104.0f) return 0.0f;
  float n = rintf(x * kLog2e);
  float r = __fmaf_rn(-n, kLn2Hi, x);
  r = __fmaf_rn(-n, kLn2Lo, r);
  float p = 1.0f / 5040.0f;
  p = __fmaf_rn(p, r, 1.0f / 720.0f);
  p = __fmaf_rn(p, r, 1.0f / 120.0f);
  p = __fmaf_rn(p, r, 1.0f / 24.0f);
  p = __fmaf_rn(p, r, 1.0f / 6.0f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int e = (int)n;
  if (e > 127)
    return __fmul_rn(__fmul_rn(p, __uint_as_float((uint32_t)(127 + 127) << 23)),
                     __uint_as_float((uint32_t)(e - 127 + 127) << 23));
  if (e < -126)
    return __fmul_rn(__fmul_rn(p, __uint_as_float((uint32_t)(e + 64 + 127) << 23)),
                     __uint_as_float((uint32_t)(-64 + 127) << 23));
  return __fmul_rn(p, __uint_as_float((uint32_t)(e + 127) << 23));
}

__device__ __forceinline__ float dlog(float x) {
  if (x != x) return x;
  if (x < 0.0f) return __int_as_float(0x7fc00000);
  if (x == 0.0f) return __int_as_float(0xff800000);
  if (x == __int_as_float(0x7f800000)) return x;
  uint32_t u = __float_as_uint(x);
  int e = 0;
  if (u < 0x00800000u) {
    u = __float_as_uint(__fmul_rn(x, 8388608.0f));
    e = -23;
  }
  e += (int)((u >> 23) & 0xffu) - 127;
  float m = __uint_as_float((u & 0x007fffffu) | 0x3f800000u);
  if (m > kSqrt2) {
    m = __fmul_rn(m, 0.5f);
    e += 1;
  }
  float f = __fsub_rn(m, 1.0f);
  float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
  float z = __fmul_rn(s, s);
  float q = 1.0f / 11.0f;
  q = __fmaf_rn(q, z, 1.0f / 9.0f);
  q = __fmaf_rn(q, z, 1.0f / 7.0f);
  q = __fmaf_rn(q, z, 1.0f / 5.0f);
  q = __fmaf_rn(q, z, 1.0f / 3.0f);
  q = __fmaf_rn(q, z, 1.0f);
  float l = __fmul_rn(__fmul_rn(2.0f, s), q);
  float fe = (float)e;
  return __fmaf_rn(fe, kLn2Hi, __fmaf_rn(fe, kLn2Lo, l));
}

// ---------------------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3",
// SC'11): counter (token, slot, offset) under key `seed` -> one 32-bit word, turned into
// log(Exp(1)) noise (per token) or an acceptance uniform (token word 0xffffffff).
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t philox_word(uint64_t seed, uint64_t offset, uint32_t slot, uint32_t token) {
  uint32_t c0 = token, c1 = slot, c2 = (uint32_t)offset, c3 = (uint32_t)(offset >> 32);
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    uint32_t hi0 = __umulhi(0xD2511F53u, c0), lo0 = 0xD2511F53u * c0;
    uint32_t hi1 = __umulhi(0xCD9E8D57u, c2), lo1 = 0xCD9E8D57u * c2;
    uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c0;
}

// a uniform draw in (0, 1): the word's top 23 bits, centred in their interval
__device__ __forceinline__ float philox_unit(uint32_t w) {
  return __fmul_rn(__fadd_rn((float)(w >> 9), 0.5f), 1.0f / 8388608.0f);
}

__device__ __forceinline__ float philox_log_exponential(uint64_t seed, uint64_t offset, uint32_t slot,
                                                        uint32_t token) {
  return dlog(-dlog(philox_unit(philox_word(seed, offset, slot, token))));
}

// acceptance uniform of a multistep slot (counter offset = the call's offset + step): the
// bf16 value of a (0, 1) draw, as the reference keeps its uniforms in bf16
__device__ __forceinline__ float philox_acceptance(uint64_t seed, uint64_t offset, uint32_t slot) {
  return rbf(philox_unit(philox_word(seed, offset, slot, 0xffffffffu)));
}

// ---------------------------------------------------------------------------------------
// warp helpers
// ---------------------------------------------------------------------------------------

template <typename T>
__device__ __forceinline__ T umax(T a, T b) { return a > b ? a : b; }
template <typename T>
__device__ __forceinline__ T umin(T a, T b) { return a < b ? a : b; }

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) v = umax(v, (uint64_t)__shfl_xor_sync(kFull, v, d));
  return v;
}

// Sum of 128 values held 4 per lane (positions 4*lane + j): lane-local left-to-right sum,
// then an xor butterfly; every lane returns the same bits.
__device__ __forceinline__ float warp_sum128(const float (&e)[4]) {
  float x = __fadd_rn(__fadd_rn(__fadd_rn(e[0], e[1]), e[2]), e[3]);
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) x = __fadd_rn(x, __shfl_xor_sync(kFull, x, d));
  return x;
}

// Inclusive prefix sums of 128 values held 4 per lane.
__device__ __forceinline__ void warp_ladder128(const float (&e)[4], float (&out)[4], int lane) {
  float p0 = e[0];
  float p1 = __fadd_rn(p0, e[1]);
  float p2 = __fadd_rn(p1, e[2]);
  float p3 = __fadd_rn(p2, e[3]);
  float s = p3;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    float y = __shfl_up_sync(kFull, s, d);
    if (lane >= d) s = __fadd_rn(s, y);
  }
  float E = __shfl_up_sync(kFull, s, 1);
  if (lane == 0) E = 0.0f;
  out[0] = __fadd_rn(E, p0);
  out[1] = __fadd_rn(E, p1);
  out[2] = __fadd_rn(E, p2);
  out[3] = __fadd_rn(E, p3);
}

// argmax over 128 values held 4 per lane, ties to the lowest position; returns the position
// (same on every lane).
__device__ __forceinline__ int warp_argmax128(const float (&v)[4], int lane) {
  float bv = v[0];
  int bi = 4 * lane;
#pragma unroll
  for (int j = 1; j < 4; ++j)
    if (v[j] > bv) {
      bv = v[j];
      bi = 4 * lane + j;
    }
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    float ov = __shfl_xor_sync(kFull, bv, d);
    int oi = __shfl_xor_sync(kFull, bi, d);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  return bi;
}

// value of position i (0..127) held 4 per lane
template <typename T>
__device__ __forceinline__ T warp_pick128(const T (&v)[4], int i) {
  T x = v[0];
#pragma unroll
  for (int j = 1; j < 4; ++j)
    if ((i & 3) == j) x = v[j];
  return __shfl_sync(kFull, x, i >> 2);
}

// Bitonic sort of 128 keys held 4 per lane (position 4*lane + j), descending.
template <typename K>
__device__ __forceinline__ void warp_sort128_desc(K (&k)[4], int lane) {
#pragma unroll
  for (int size = 2; size <= 128; size <<= 1) {
#pragma unroll
    for (int d = size >> 1; d >= 1; d >>= 1) {
      if (d >= 4) {
        const int ld = d >> 2;
        const bool lower = (lane & ld) == 0;
        const bool desc = ((4 * lane) & size) == 0;
        const bool keep_max = (lower == desc);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          K o = __shfl_xor_sync(kFull, k[j], ld);
          k[j] = keep_max ? umax(k[j], o) : umin(k[j], o);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if ((j & d) == 0) {
            const int i = 4 * lane + j;
            const bool desc = (i & size) == 0;
            K a = k[j], b = k[j | d];
            K mx = umax(a, b), mn = umin(a, b);
            k[j] = desc ? mx : mn;
            k[j | d] = desc ? mn : mx;
          }
        }
      }
    }
  }
}

// a := top-128 of (a U b), both descending-sorted, result descending-sorted.
template <typename K>
__device__ __forceinline__ void warp_merge128_desc(K (&a)[4], const K (&b)[4], int lane) {
  // reverse b: position i <- 127 - i  (lane 31-lane, slot 3-j)
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    K r = __shfl_sync(kFull, b[3 - j], 31 - lane);
    a[j] = umax(a[j], r);
  }
  // bitonic half-cleaners, descending
#pragma unroll
  for (int d = 64; d >= 4; d >>= 1) {
    const int ld = d >> 2;
    const bool lower = (lane & ld) == 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      K o = __shfl_xor_sync(kFull, a[j], ld);
      a[j] = lower ? umax(a[j], o) : umin(a[j], o);
    }
  }
#pragma unroll
  for (int d = 2; d >= 1; d >>= 1) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if ((j & d) == 0) {
        K x = a[j], y = a[j | d];
        a[j] = umax(x, y);
        a[j | d] = umin(x, y);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// packed bf16x2 arithmetic (round-to-nearest-even, one rounding per operation, exactly as
// the reference's bf16 operations round)
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// {lo, hi} fp32 -> packed bf16x2 (lo in bits 0..15), round to nearest even
__device__ __forceinline__ uint32_t bf2_pack(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

__device__ __forceinline__ float bf2_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf2_hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

// ---------------------------------------------------------------------------------------
// bulk (TMA) global -> shared copies completed on an mbarrier; every CTA loads its own data.
// ---------------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

// more bytes for the current phase without an arrival (the arrival comes with a later
// mbar_expect_tx or mbar_arrive)
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar`, giving up after `limit` polls (each poll may suspend
// the thread for a hardware-defined interval). Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// order this thread's earlier generic-proxy shared-memory accesses before later async-proxy
// (bulk copy) writes to the same shared memory
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

}  // namespace sonic
