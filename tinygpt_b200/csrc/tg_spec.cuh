// tg_spec.cuh -- speculative-decoding verification (rejection sampling).
//
// Reference: native-mac/Sources/TinyGPT/SpeculativeDecode.swift:121-210
// (stochastic, Leviathan et al.) and :41-98 (greedy).  The reference walks the
// K positions on the host with two softmaxes and several device->host reads per
// position; here two kernels do the whole batch:
//   spec_stats_kernel  one CTA per (row, position, target|draft) vocab row:
//                      max s = max x / T and the exact mass sum Z = sum q, plus
//                      the first argmax (greedy rows).  One HBM pass for the
//                      max, the second pass hits L2 (the row was just read).
//   spec_verify_kernel one CTA per batch row: the sequential accept chain from
//                      the stats, then the final draw (residual, target or bonus)
//                      by an index-ordered chunked inverse CDF over the vocab.
#pragma once

#include "../../include/tgsample.h"
#include "tg_block.cuh"

namespace tg {

constexpr int kSpecNT = 512;

struct __align__(16) SpecStat {
  float smax;
  int argmax;
  unsigned long long Z;
};

struct SpecArgs {
  const void* target;
  const void* draft;
  int32_t batch;
  int32_t K;
  int32_t vocab;
  const int32_t* draft_ids;
  const float* temperature;
  const float* u_accept;
  const float* u_draw;
  int32_t* out_ids;
  int32_t* out_n;
  SpecStat* stats;  // [batch, 2K+1]
  uint32_t* status;
};

__device__ __forceinline__ float spec_T(float t0) { return fmaxf(t0, 1e-5f); }

// Visit every element of a vocab row: 128-bit loads over the aligned middle,
// scalar loads for the unaligned head and tail.  f(v, x) per element.
template <int DT, int NT, class F>
__device__ __forceinline__ void row_for_each(const void* rowv, int V, F&& f) {
  using E = Elt<DT>;
  constexpr int EPV = E::kEPV;
  const char* row = reinterpret_cast<const char*>(rowv);
  const uintptr_t addr = reinterpret_cast<uintptr_t>(row);
  int head = static_cast<int>(((16u - (addr & 15u)) & 15u) / E::kSize);
  if (head > V) head = V;
  const int nvec = (V - head) / EPV;
  const int tail0 = head + nvec * EPV;
  const uint4* vrow = reinterpret_cast<const uint4*>(row + head * E::kSize);
  const int t = threadIdx.x;
  if (t < head) f(t, E::load(row, t));
  if (t < V - tail0) f(tail0 + t, E::load(row, tail0 + t));
  for (int jb = 0; jb < nvec; jb += 4 * NT) {
    uint4 w[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int j = jb + q * NT + t;
      if (j < nvec) w[q] = ldg_stream(vrow + j);
    }
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int j = jb + q * NT + t;
      if (j < nvec) {
        float x[EPV];
        E::unpack(w[q], x);
#pragma unroll
        for (int e = 0; e < EPV; e++) f(head + j * EPV + e, x[e]);
      }
    }
  }
}

template <int DT>
__global__ void __launch_bounds__(kSpecNT) spec_stats_kernel(SpecArgs a) {
  __shared__ BlockScratch sm;
  const int P = 2 * a.K + 1;
  const int r = blockIdx.x;
  const int b = r / P, pos = r % P;
  const int V = a.vocab;
  const float t0 = a.temperature[b];
  const bool greedy = !(t0 > 0.0f);
  const void* row;
  if (pos <= a.K) {
    row = reinterpret_cast<const char*>(a.target) +
          (static_cast<int64_t>(b) * (a.K + 1) + pos) * V * Elt<DT>::kSize;
  } else {
    if (greedy) return;
    row = reinterpret_cast<const char*>(a.draft) +
          (static_cast<int64_t>(b) * a.K + (pos - a.K - 1)) * V * Elt<DT>::kSize;
  }
  float y = neg_inf();
  int id = 0x7fffffff;
  row_for_each<DT, kSpecNT>(row, V, [&](int v, float x) {
    if (x > y || (x == y && v < id)) { y = x; id = v; }
  });
  block_argmax<kSpecNT>(y, id, sm);
  if (greedy) {
    if (threadIdx.x == 0) a.stats[r] = SpecStat{y, id, 0ull};
    return;
  }
  const float T = spec_T(t0);
  const float smax = __fdiv_rn(y, T);
  unsigned long long Z = 0;
  row_for_each<DT, kSpecNT>(row, V, [&](int, float x) {
    Z += qmass(__fsub_rn(__fdiv_rn(x, T), smax));
  });
  Z = block_sum<kSpecNT>(Z, sm);
  if (threadIdx.x == 0) a.stats[r] = SpecStat{smax, id, Z};
}

// Residual mass of one token: trunc(max(0, qT/ZT - qD/ZD) * 2^52).
__device__ __forceinline__ unsigned long long resid_mass(unsigned long long qT, double ZT,
                                                         unsigned long long qD, double ZD) {
  const double d = __dsub_rn(__ddiv_rn(__ull2double_rn(qT), ZT), __ddiv_rn(__ull2double_rn(qD), ZD));
  return d > 0.0 ? __double2ull_rz(__dmul_rn(d, kResidScale)) : 0ull;
}

template <int DT>
__global__ void __launch_bounds__(kSpecNT) spec_verify_kernel(SpecArgs a) {
  using E = Elt<DT>;
  __shared__ BlockScratch sm;
  __shared__ int s_final;  // -1: all accepted (bonus), else the rejecting position
  __shared__ int s_n;
  const int b = blockIdx.x;
  const int K = a.K, V = a.vocab, P = 2 * K + 1;
  const float t0 = a.temperature[b];
  const bool greedy = !(t0 > 0.0f);
  const float T = spec_T(t0);
  const SpecStat* st = a.stats + static_cast<int64_t>(b) * P;
  int32_t* out = a.out_ids + static_cast<int64_t>(b) * (K + 1);
  const char* tgt = reinterpret_cast<const char*>(a.target) + static_cast<int64_t>(b) * (K + 1) * V * E::kSize;
  const char* drf = greedy ? nullptr : reinterpret_cast<const char*>(a.draft) + static_cast<int64_t>(b) * K * V * E::kSize;

  if (threadIdx.x == 0) {
    for (int i = 0; i <= K; i++) out[i] = -1;
    int n = 0, fin = -1;
    for (int i = 0; i < K; i++) {
      const int tok = a.draft_ids[static_cast<int64_t>(b) * K + i];
      if (greedy) {
        const int am = st[i].argmax;
        if (am == tok) { out[n++] = tok; continue; }
        out[n++] = am;
        fin = -2;  // done, nothing to draw
        break;
      }
      bool accept = false;
      if (tok >= 0 && tok < V) {
        const unsigned long long qT = qmass(__fsub_rn(__fdiv_rn(E::load(tgt + static_cast<int64_t>(i) * V * E::kSize, tok), T), st[i].smax));
        const unsigned long long qD = qmass(__fsub_rn(__fdiv_rn(E::load(drf + static_cast<int64_t>(i) * V * E::kSize, tok), T), st[K + 1 + i].smax));
        const double pT = __ddiv_rn(__ull2double_rn(qT), __ull2double_rn(st[i].Z));
        const double pD = __ddiv_rn(__ull2double_rn(qD), __ull2double_rn(st[K + 1 + i].Z));
        const double ratio = __ddiv_rn(pT, pD > 1e-10 ? pD : 1e-10);
        const double lim = ratio < 1.0 ? ratio : 1.0;
        accept = static_cast<double>(a.u_accept[static_cast<int64_t>(b) * K + i]) <= lim;
      } else {
        atomicOr(a.status, 2u);
      }
      if (accept) { out[n++] = tok; continue; }
      fin = i;
      break;
    }
    if (greedy && fin == -1) {
      out[n++] = st[K].argmax;
      fin = -2;
    }
    s_final = fin;
    s_n = n;
  }
  __syncthreads();
  const int fin = s_final;
  if (fin == -2) {
    if (threadIdx.x == 0) a.out_n[b] = s_n;
    return;
  }

  // Final draw over the vocab in index order.  Thread t owns the contiguous
  // chunk [t*C, t*C+C); chunk sums -> block scan -> the owning thread rescans.
  const int pos = fin < 0 ? K : fin;
  const char* trow = tgt + static_cast<int64_t>(pos) * V * E::kSize;
  const char* drow = fin < 0 ? nullptr : drf + static_cast<int64_t>(fin) * V * E::kSize;
  const float smT = st[pos].smax;
  const double ZT = __ull2double_rn(st[pos].Z);
  const float smD = fin < 0 ? 0.0f : st[K + 1 + fin].smax;
  const double ZD = fin < 0 ? 1.0 : __ull2double_rn(st[K + 1 + fin].Z);
  const int C = (V + kSpecNT - 1) / kSpecNT;
  const int v0 = threadIdx.x * C;
  const int v1 = min(V, v0 + C);
  auto qt_of = [&](int v) { return qmass(__fsub_rn(__fdiv_rn(E::load(trow, v), T), smT)); };
  auto rq_of = [&](int v) {
    const unsigned long long qd = qmass(__fsub_rn(__fdiv_rn(E::load(drow, v), T), smD));
    return resid_mass(qt_of(v), ZT, qd, ZD);
  };
  bool use_resid = false;
  unsigned long long csum = 0, total = 0;
  if (fin >= 0) {
    for (int v = v0; v < v1; v++) csum += rq_of(v);
    unsigned long long R;
    block_excl_scan<kSpecNT>(csum, R, sm);
    use_resid = __dmul_rn(__ull2double_rn(R), 1.0 / kResidScale) > 1e-10;
  }
  if (!use_resid) {
    csum = 0;
    for (int v = v0; v < v1; v++) csum += qt_of(v);
  }
  const unsigned long long before = block_excl_scan<kSpecNT>(csum, total, sm);
  const unsigned long long r = draw_point(a.u_draw[b], total);
  if (csum > 0 && before <= r && r < before + csum) {
    unsigned long long c = before;
    int pick = v1 - 1;
    for (int v = v0; v < v1; v++) {
      c += use_resid ? rq_of(v) : qt_of(v);
      if (c > r) { pick = v; break; }
    }
    out[s_n] = pick;
    a.out_n[b] = s_n + 1;
  }
}

}  // namespace tg
