// tg_common.cuh -- arithmetic shared by every kernel of the sampling engine.
//
// The sampling semantics are defined operation by operation (include/tgsample.h)
// so the GPU result is reproducible bit for bit on a CPU.  Every floating-point
// step below is one correctly rounded IEEE operation written as an intrinsic, so
// neither contraction nor fast-math can change it.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace tg {

constexpr float kMassScale = 17592186044416.0f;  // 2^44: fixed-point scale of masses
constexpr double kResidScale = 4503599627370496.0;  // 2^52: scale of residual masses

// exp(x): Cody-Waite reduction x = n*ln2 + r with |r| <= ln2/2 (ln2 split in a
// 16-bit head and a tail), the degree-7 Taylor polynomial of e^r in Horner form
// (truncation error < 6e-9 relative), then an exact scaling by 2^n done as one
// or two multiplications by powers of two.  Accuracy < 1 ulp over the normal
// range (checked against libm in the tests).  Independent of CUDA's expf.
// The reduction and the polynomial: x = n*ln2 + r, p = e^r.
// n = rint(x * log2(e)) without the conversion pipe: for |p| < 2^22, adding
// 1.5 * 2^23 puts p + 1.5 * 2^23 in [2^23, 2^24), where the spacing of floats is
// 1, so the correctly rounded sum is p rounded to an integer, ties to even (the
// constant is even), exactly rintf(p); its bits minus the constant's bits are
// that integer.  Every x used here gives |p| < 151 (tg_exp returns early
// outside (-104, 88]; qmass_le0 discards d < -32, whatever ni is then).
__device__ __forceinline__ float tg_exp_poly(float x, int& ni) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23, bits 0x4B400000
  const float tr = __fadd_rn(__fmul_rn(x, 1.44269504088896341f), kRound);
  const float n = __fsub_rn(tr, kRound);
  float r = __fmaf_rn(n, -0.693145751953125f, x);
  r = __fmaf_rn(n, -1.42860676533018e-06f, r);
  float p = 1.98412698412698e-04f;
  p = __fmaf_rn(p, r, 1.38888888888889e-03f);
  p = __fmaf_rn(p, r, 8.33333333333333e-03f);
  p = __fmaf_rn(p, r, 4.16666666666667e-02f);
  p = __fmaf_rn(p, r, 1.66666666666667e-01f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  ni = __float_as_int(tr) - 0x4B400000;
  return p;
}

__device__ __forceinline__ float tg_exp(float x) {
  if (!(x > -104.0f)) return 0.0f;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  int ni;
  float p = tg_exp_poly(x, ni);
  if (ni >= -126) return __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(ni + 127) << 23));
  p = __fmul_rn(p, __uint_as_float(1u << 23));
  return __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(ni + 126 + 127) << 23));
}

// Fixed-point mass of a tempered logit d = s - max(s) <= 0.
__device__ __forceinline__ uint64_t qmass(float d) {
  if (!(d >= -32.0f)) return 0ull;
  return __float2ull_rz(__fmul_rn(tg_exp(d), kMassScale));
}

// qmass(d) for d <= 0 without branches: for -32 <= d <= 0 tg_exp takes its
// first scaling branch (n >= -47), and both of qmass's scalings (by 2^n, then
// by 2^44) are exact there (normal results), so one multiplication by
// 2^(n + 44) gives the same bits; below -32 (or NaN) the select gives 0.
__device__ __forceinline__ uint64_t qmass_le0(float d) {
  int ni;
  const float p = tg_exp_poly(d, ni);
  const float e44 = __fmul_rn(p, __uint_as_float((static_cast<uint32_t>(ni) + 171u) << 23));
  const uint64_t q = __float2ull_rz(e44);
  return d >= -32.0f ? q : 0ull;
}

// Hash of a token id for the history tables: the 32-bit finaliser of
// MurmurHash3 (fmix32), so every id bit reaches every hash bit.  A plain
// multiplicative hash maps ids in arithmetic progression (an affine token
// permutation, a tokenizer's id blocks) onto runs of neighbouring slots, and
// linear probing then walks those runs on every lookup.
__device__ __forceinline__ uint32_t tg_mix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}

// Order-preserving 32-bit key of a float (-0 folded onto +0).
__device__ __forceinline__ uint32_t fkey(float x) {
  const uint32_t u = __float_as_uint(x == 0.0f ? 0.0f : x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ float neg_inf() { return __int_as_float(0xff800000); }

// r = trunc(u * total) clamped to [0, total); a NaN or negative u counts as 0.
__device__ __forceinline__ uint64_t draw_point(float u, uint64_t total) {
  if (!(u >= 0.0f)) u = 0.0f;
  uint64_t r = __double2ull_rz(__dmul_rn(static_cast<double>(u), __ull2double_rn(total)));
  return r >= total ? total - 1 : r;
}

// bf16 bit pattern -> fp32 (exact).
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Shared-memory address of a generic pointer into shared memory.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 128-bit streaming load that bypasses L1 (data is read once per row).
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

template <int DT>
struct Elt;

template <>
struct Elt<1> {  // bf16
  static constexpr int kEPV = 8;
  static constexpr int kSize = 2;
  __device__ __forceinline__ static void unpack(const uint4& w, float* x) {
    x[0] = bf16_lo(w.x); x[1] = bf16_hi(w.x);
    x[2] = bf16_lo(w.y); x[3] = bf16_hi(w.y);
    x[4] = bf16_lo(w.z); x[5] = bf16_hi(w.z);
    x[6] = bf16_lo(w.w); x[7] = bf16_hi(w.w);
  }
  __device__ __forceinline__ static float load(const void* row, int64_t i) {
    const uint16_t h = __ldg(reinterpret_cast<const unsigned short*>(row) + i);
    return __uint_as_float(static_cast<uint32_t>(h) << 16);
  }
  // max of the 8 values (packed bf16x2 maxima, then one fp32 max)
  __device__ __forceinline__ static float vmax(const uint4& w) {
    uint32_t a, b, m;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(a) : "r"(w.x), "r"(w.y));
    asm("max.bf16x2 %0, %1, %2;" : "=r"(b) : "r"(w.z), "r"(w.w));
    asm("max.bf16x2 %0, %1, %2;" : "=r"(m) : "r"(a), "r"(b));
    return fmaxf(bf16_lo(m), bf16_hi(m));
  }
  // max over N vectors: a packed bf16x2 tree, one fp32 max at the end
  template <int N>
  __device__ __forceinline__ static float vmax_n(const uint4* w) {
    uint32_t r[2 * N];
#pragma unroll
    for (int q = 0; q < N; q++) {
      asm("max.bf16x2 %0, %1, %2;" : "=r"(r[2 * q]) : "r"(w[q].x), "r"(w[q].y));
      asm("max.bf16x2 %0, %1, %2;" : "=r"(r[2 * q + 1]) : "r"(w[q].z), "r"(w[q].w));
    }
#pragma unroll
    for (int n = 2 * N; n > 1; n >>= 1) {
#pragma unroll
      for (int i = 0; i < n / 2; i++) asm("max.bf16x2 %0, %1, %2;" : "=r"(r[i]) : "r"(r[2 * i]), "r"(r[2 * i + 1]));
    }
    return fmaxf(bf16_lo(r[0]), bf16_hi(r[0]));
  }
};

template <>
struct Elt<0> {  // fp32
  static constexpr int kEPV = 4;
  static constexpr int kSize = 4;
  __device__ __forceinline__ static void unpack(const uint4& w, float* x) {
    x[0] = __uint_as_float(w.x); x[1] = __uint_as_float(w.y);
    x[2] = __uint_as_float(w.z); x[3] = __uint_as_float(w.w);
  }
  __device__ __forceinline__ static float load(const void* row, int64_t i) {
    return __ldg(reinterpret_cast<const float*>(row) + i);
  }
  __device__ __forceinline__ static float vmax(const uint4& w) {
    return fmaxf(fmaxf(__uint_as_float(w.x), __uint_as_float(w.y)),
                 fmaxf(__uint_as_float(w.z), __uint_as_float(w.w)));
  }
  template <int N>
  __device__ __forceinline__ static float vmax_n(const uint4* w) {
    float m = vmax(w[0]);
#pragma unroll
    for (int q = 1; q < N; q++) m = fmaxf(m, vmax(w[q]));
    return m;
  }
};

// Bits e0 .. e0+n-1 (n <= 8) of a bitmask row, bit i of the result = token e0+i.
__device__ __forceinline__ uint32_t mask_bits(const uint32_t* m, int e0, int n) {
  const int w = e0 >> 5, sh = e0 & 31;
  const uint32_t lo = __ldg(m + w);
  const uint32_t hi = (sh + n > 32) ? __ldg(m + w + 1) : 0u;
  return __funnelshift_r(lo, hi, sh) & ((1u << n) - 1u);
}

__device__ __forceinline__ bool mask_allows(const uint32_t* m, int v) {
  return (__ldg(m + (v >> 5)) >> (v & 31)) & 1u;
}

}  // namespace tg
