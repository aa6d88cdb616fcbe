// tg_spec.cuh -- speculative-decoding verification (rejection sampling).
//
// Reference: native-mac/Sources/TinyGPT/SpeculativeDecode.swift:121-210
// (stochastic, Leviathan et al.) and :41-98 (greedy).  The reference walks the
// K positions on the host with two softmaxes and several device->host reads per
// position; here two cluster kernels do the whole batch:
//   spec_stats_kernel   one 8-CTA cluster per (row, position, target|draft) vocab
//                       row.  Each CTA streams its slice of the row from HBM
//                       once (maximum; lines kept in L2 with an evict_last
//                       policy) and re-reads it from L2 for the exact mass sum
//                       Z = sum q; the slice results are combined over
//                       distributed shared memory.
//   spec_verify_kernel  one 8-CTA cluster per batch row.  Rank 0 runs the
//                       sequential accept chain; every CTA sums the final
//                       distribution's masses over its slice; the slice sums,
//                       exchanged over DSMEM, locate the slice holding the draw
//                       point, whose CTA finds the id with an ordered scan.
#pragma once

#include <cooperative_groups.h>

#include "../../include/tgsample.h"
#include "tg_block.cuh"

namespace tg {

namespace cg = cooperative_groups;

constexpr int kSpecNT = 256;
constexpr int kSpecCluster = 8;
#ifndef TG_VERIFY_MINB
#define TG_VERIFY_MINB 4
#endif
constexpr int kVerifyMinCtas = TG_VERIFY_MINB;  // verify kernel occupancy target (registers <= 64)

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
  int32_t chunk;    // elements per cluster rank (multiple of 8)
  // lazy mode: positions are evaluated one at a time for the rows still
  // accepting; rstate[2b] = accepted count, rstate[2b+1] = -1 while accepting,
  // the rejecting position, or -2 when the row is finished (greedy)
  int32_t* rstate;  // nullptr: eager (every position at once)
  int32_t lazy_pos; // position of this lazy stats launch (K: the bonus row)
  // grammar masks (tg_spec_verify_masked): state_ids [batch, K+1], the state
  // before each position's token (-1: unmasked); nullptr: no masks
  const uint32_t* mask_table;
  int32_t num_states;
  int32_t mask_words;
  const int32_t* state_ids;
};

// Mask row of position i of batch row b (nullptr: unmasked).  An out-of-range
// state leaves the position unmasked and sets status bit 0.
__device__ __forceinline__ const uint32_t* spec_mask(const SpecArgs& a, int b, int i) {
  if (!a.state_ids) return nullptr;
  const int sid = a.state_ids[static_cast<int64_t>(b) * (a.K + 1) + i];
  if (sid < 0) return nullptr;
  if (sid >= a.num_states) {
    atomicOr(a.status, 1u);
    return nullptr;
  }
  return a.mask_table + static_cast<int64_t>(sid) * a.mask_words;
}

__device__ __forceinline__ float spec_T(float t0) { return fmaxf(t0, 1e-5f); }

// 128-bit load with an L2 eviction policy (createpolicy): the statistics
// kernel streams its slice from HBM once keeping the lines (evict_last), then
// re-reads them from L2 for the masses and lets them go (evict_first).
template <bool kKeep>
__device__ __forceinline__ uint4 ld_l2hint(const uint4* p) {
  uint4 v;
  if constexpr (kKeep) {
    asm volatile(
        "{ .reg .b64 pol; createpolicy.fractional.L2::evict_last.b64 pol, 1.0;"
        " ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], pol; }"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
  } else {
    asm volatile(
        "{ .reg .b64 pol; createpolicy.fractional.L2::evict_first.b64 pol, 1.0;"
        " ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], pol; }"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
  }
  return v;
}

constexpr int kSpecLoads = 4;  // 16-byte loads in flight per thread

// Visit elements [0, n) of a slice at `src` (global memory): f(i, x) for each,
// x = -inf where the mask row `msk` (bit c0 + i) clears it.  A thread visits
// its elements in increasing index order.  The 16-byte-aligned body goes as
// kSpecLoads vectors in flight per thread; the rest element by element.
template <int DT, bool kKeep, class F>
__device__ __forceinline__ void slice_for_each(const char* src, int n, int c0, const uint32_t* msk, F&& f) {
  using E = Elt<DT>;
  constexpr int EPV = E::kEPV;
  const int t = threadIdx.x;
  const int nv = (reinterpret_cast<uintptr_t>(src) & 15u) == 0 ? n / EPV : 0;
  const uint4* sv = reinterpret_cast<const uint4*>(src);
  for (int j0 = 0; j0 < nv; j0 += kSpecLoads * kSpecNT) {
    uint4 w[kSpecLoads];
#pragma unroll
    for (int q = 0; q < kSpecLoads; q++) {
      const int j = j0 + q * kSpecNT + t;
      if (j < nv) w[q] = ld_l2hint<kKeep>(sv + j);
    }
#pragma unroll
    for (int q = 0; q < kSpecLoads; q++) {
      const int j = j0 + q * kSpecNT + t;
      if (j >= nv) break;
      float x[EPV];
      E::unpack(w[q], x);
      const uint32_t bits = msk ? mask_bits(msk, c0 + j * EPV, EPV) : 0xffu;
#pragma unroll
      for (int e = 0; e < EPV; e++) f(j * EPV + e, ((bits >> e) & 1u) ? x[e] : neg_inf());
    }
  }
  for (int i = nv * EPV + t; i < n; i += kSpecNT) {
    const float x = E::load(src, i);
    f(i, (msk && !mask_allows(msk, c0 + i)) ? neg_inf() : x);
  }
}

// Statistics of one vocab row on an 8-CTA cluster, each CTA one slice.  Pass 1
// streams the slice from HBM (maximum, first argmax); the cluster combines the
// slice maxima over distributed shared memory; pass 2 re-reads the slice from
// L2 for the exact mass sum Z.  No shared-memory staging: occupancy is set by
// registers, so CTAs of different rows overlap their HBM streams with other
// CTAs' mass arithmetic.
template <int DT, bool kMask>
__global__ void __cluster_dims__(kSpecCluster, 1, 1) __launch_bounds__(kSpecNT, 4)
    spec_stats_kernel(SpecArgs a) {
  using E = Elt<DT>;
  // launched as a programmatic dependent: the previous launch of the chain
  // (statistics, accept tests) must be complete before anything is read
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ ReduceScratch sm;
  __shared__ float c_max;
  __shared__ int c_arg;
  __shared__ unsigned long long c_z;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int t = threadIdx.x;
  const int P = 2 * a.K + 1;
  int b, pos;
  if (!a.rstate) {  // eager: every (row, position) at once
    b = (blockIdx.x / kSpecCluster) / P;
    pos = (blockIdx.x / kSpecCluster) % P;
  } else if (a.lazy_pos < a.K) {  // lazy: target and draft rows of one position
    const int rl = blockIdx.x / kSpecCluster;
    b = rl >> 1;
    pos = (rl & 1) ? a.K + 1 + a.lazy_pos : a.lazy_pos;
    if (a.lazy_pos > 0 && a.rstate[2 * b + 1] != -1) return;  // the whole cluster
  } else {  // lazy: the bonus row of the rows that accepted every proposal
    b = blockIdx.x / kSpecCluster;
    pos = a.K;
    if (a.K > 0 && a.rstate[2 * b + 1] != -1) return;
  }
  const int r = b * P + pos;
  const int V = a.vocab;
  const float t0 = a.temperature[b];
  const bool greedy = !(t0 > 0.0f);
  // the whole cluster: the draft row is not needed (greedy row, or a call
  // without draft logits)
  if (pos > a.K && (greedy || !a.draft)) return;
  const char* row;
  if (pos <= a.K) {
    row = reinterpret_cast<const char*>(a.target) + (static_cast<int64_t>(b) * (a.K + 1) + pos) * V * E::kSize;
  } else {
    row = reinterpret_cast<const char*>(a.draft) + (static_cast<int64_t>(b) * a.K + (pos - a.K - 1)) * V * E::kSize;
  }
  const int c0 = min(V, rank * a.chunk), c1 = min(V, c0 + a.chunk);
  const char* src = row + static_cast<int64_t>(c0) * E::kSize;
  const uint32_t* msk = !kMask ? nullptr : spec_mask(a, b, pos <= a.K ? pos : pos - a.K - 1);
  // pass 1: maximum and its first index (`x > y` keeps the first)
  float y = neg_inf();
  int id = 0x7fffffff;
  auto amax = [&](int i, float x) {
    if (x > y) { y = x; id = c0 + i; }
  };
  if (greedy) slice_for_each<DT, false>(src, c1 - c0, c0, msk, amax);  // read once: no need to keep
  else slice_for_each<DT, true>(src, c1 - c0, c0, msk, amax);
  block_argmax<kSpecNT>(y, id, sm);
  if (t == 0) { c_max = y; c_arg = id; }
  cluster.sync();
  for (int q = 0; q < kSpecCluster; q++) {
    const float oy = *cluster.map_shared_rank(&c_max, q);
    const int oi = *cluster.map_shared_rank(&c_arg, q);
    if (q == 0 || oy > y || (oy == y && oi < id)) { y = oy; id = oi; }
  }
  if (msk && id == 0x7fffffff) id = -1;  // nothing allowed above -inf
  if (greedy) {
    if (rank == 0 && t == 0) a.stats[r] = SpecStat{y, id, 0ull};
    cluster.sync();  // peers still read this CTA's maximum
    return;
  }
  const float T = spec_T(t0);
  const float smax = __fdiv_rn(y, T);
  // pass 2: the exact masses (d = x / T - smax <= 0: the branch-free form)
  unsigned long long Z = 0;
  slice_for_each<DT, false>(src, c1 - c0, c0, msk, [&](int, float x) {
    Z += qmass_le0(__fsub_rn(__fdiv_rn(x, T), smax));
  });
  Z = block_sum<kSpecNT>(Z, sm);
  if (t == 0) c_z = Z;
  cluster.sync();
  if (rank == 0 && t == 0) {
    unsigned long long tot = 0;
    for (int q = 0; q < kSpecCluster; q++) tot += *cluster.map_shared_rank(&c_z, q);
    a.stats[r] = SpecStat{smax, id, tot};
  }
  cluster.sync();  // peers still read this CTA's sum
}

// Residual mass of one token: trunc(max(0, qT/ZT - qD/ZD) * 2^52).
__device__ __forceinline__ unsigned long long resid_mass(unsigned long long qT, double ZT,
                                                         unsigned long long qD, double ZD) {
  const double d = __dsub_rn(__ddiv_rn(__ull2double_rn(qT), ZT), __ddiv_rn(__ull2double_rn(qD), ZD));
  return d > 0.0 ? __double2ull_rz(__dmul_rn(d, kResidScale)) : 0ull;
}

// resid_mass with an exact early-out: when qT / ZT <= qD / ZD as real numbers
// (qT * ZD <= qD * ZT in 128-bit integers; ZT and ZD hold integer values, ZTi
// and ZDi are the same integers), the rounded quotients keep that order, the
// difference is <= 0 and the residual is 0 -- the divisions are skipped.
__device__ __forceinline__ unsigned long long resid_mass_x(unsigned long long qT, double ZT,
                                                           unsigned long long ZTi, unsigned long long qD,
                                                           double ZD, unsigned long long ZDi) {
  const unsigned long long h1 = __umul64hi(qT, ZDi), l1 = qT * ZDi;
  const unsigned long long h2 = __umul64hi(qD, ZTi), l2 = qD * ZTi;
  if (h1 < h2 || (h1 == h2 && l1 <= l2)) return 0ull;
  return resid_mass(qT, ZT, qD, ZD);
}

// One accept test of batch row b at position i (thread-level): appends to out
// and sets fin to i on a stochastic reject, -2 on a greedy mismatch.
template <int DT, bool kMask>
__device__ __forceinline__ void spec_accept_step(const SpecArgs& a, int b, int i, int32_t* out,
                                                 int& n, int& fin) {
  using E = Elt<DT>;
  const int K = a.K, V = a.vocab, P = 2 * K + 1;
  const float t0 = a.temperature[b];
  const bool greedy = !(t0 > 0.0f);
  const float T = spec_T(t0);
  const SpecStat* st = a.stats + static_cast<int64_t>(b) * P;
  const int tok = a.draft_ids[static_cast<int64_t>(b) * K + i];
  if (greedy) {
    const int am = st[i].argmax;
    out[n++] = am;
    if (am != tok) fin = -2;
    return;
  }
  if (!a.draft) {  // draft-free call: a stochastic row ends without a token
    atomicOr(a.status, 16u);
    fin = -2;
    return;
  }
  bool accept = false;
  const uint32_t* msk = !kMask ? nullptr : spec_mask(a, b, i);
  if (tok >= 0 && tok < V && msk && !mask_allows(msk, tok)) {
    // a proposal the grammar does not allow is rejected
  } else if (tok >= 0 && tok < V) {
    const char* trow = reinterpret_cast<const char*>(a.target) + (static_cast<int64_t>(b) * (K + 1) + i) * V * E::kSize;
    const char* drow = reinterpret_cast<const char*>(a.draft) + (static_cast<int64_t>(b) * K + i) * V * E::kSize;
    const unsigned long long qT = qmass_le0(__fsub_rn(__fdiv_rn(E::load(trow, tok), T), st[i].smax));
    const unsigned long long qD = qmass_le0(__fsub_rn(__fdiv_rn(E::load(drow, tok), T), st[K + 1 + i].smax));
    const double pT = __ddiv_rn(__ull2double_rn(qT), __ull2double_rn(st[i].Z));
    const double pD = __ddiv_rn(__ull2double_rn(qD), __ull2double_rn(st[K + 1 + i].Z));
    const double ratio = __ddiv_rn(pT, pD > 1e-10 ? pD : 1e-10);
    const double lim = ratio < 1.0 ? ratio : 1.0;
    accept = static_cast<double>(a.u_accept[static_cast<int64_t>(b) * K + i]) <= lim;
  } else {
    atomicOr(a.status, 2u);
  }
  if (accept) out[n++] = tok;
  else fin = i;
}

// Lazy mode: position i of every row still accepting, one thread per row.
template <int DT, bool kMask>
__global__ void __launch_bounds__(128) spec_chain_kernel(SpecArgs a, int i) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the statistics of position i
  const int b = blockIdx.x * 128 + threadIdx.x;
  if (b >= a.batch) return;
  int32_t* out = a.out_ids + static_cast<int64_t>(b) * (a.K + 1);
  int n = 0, fin = -1;
  if (i == 0) {
    for (int j = 0; j <= a.K; j++) out[j] = -1;
  } else {
    n = a.rstate[2 * b];
    fin = a.rstate[2 * b + 1];
    if (fin != -1) return;
  }
  spec_accept_step<DT, kMask>(a, b, i, out, n, fin);
  a.rstate[2 * b] = n;
  a.rstate[2 * b + 1] = fin;
}

template <int DT, bool kMask>
__global__ void __cluster_dims__(kSpecCluster, 1, 1) __launch_bounds__(kSpecNT, kVerifyMinCtas)
    spec_verify_kernel(SpecArgs a) {
  using E = Elt<DT>;
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the last statistics / accept launch
  __shared__ ReduceScratch sm;
  __shared__ int s_fin, s_n;  // rank 0: the rejecting position (-1 bonus, -2 done) and accepted count
  __shared__ unsigned long long c_sumT, c_sumR;
  __shared__ int s_ent;                  // the table entry holding the draw point
  __shared__ unsigned long long s_before;  // mass before that entry
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int t = threadIdx.x;
  const int b = blockIdx.x / kSpecCluster;
  const int K = a.K, V = a.vocab, P = 2 * K + 1;
  const float t0 = a.temperature[b];
  const bool greedy = !(t0 > 0.0f);
  const float T = spec_T(t0);
  const SpecStat* st = a.stats + static_cast<int64_t>(b) * P;
  int32_t* out = a.out_ids + static_cast<int64_t>(b) * (K + 1);
  const char* tgt = reinterpret_cast<const char*>(a.target) + static_cast<int64_t>(b) * (K + 1) * V * E::kSize;
  const char* drf = (greedy || !a.draft) ? nullptr : reinterpret_cast<const char*>(a.draft) + static_cast<int64_t>(b) * K * V * E::kSize;

  if (rank == 0 && t == 0) {
    int n = 0, fin = -1;
    if (!a.rstate) {
      for (int i = 0; i <= K; i++) out[i] = -1;
      for (int i = 0; i < K && fin == -1; i++) spec_accept_step<DT, kMask>(a, b, i, out, n, fin);
    } else if (K == 0) {
      out[0] = -1;
    } else {
      n = a.rstate[2 * b];
      fin = a.rstate[2 * b + 1];
    }
    if (greedy && fin == -1) {  // every proposal matched: the bonus is the target argmax
      out[n++] = st[K].argmax;
      fin = -2;
    }
    s_fin = fin;
    s_n = n;
  }
  cluster.sync();
  const int fin = *cluster.map_shared_rank(&s_fin, 0);
  const int n0 = *cluster.map_shared_rank(&s_n, 0);
  if (fin == -2) {
    if (rank == 0 && t == 0) a.out_n[b] = n0;
    cluster.sync();
    return;
  }

  // Final draw over the vocab in index order.  The CTA's slice [c0, c1) is cut
  // into tiles of kSpecNT * EPV elements; thread t takes the EPV consecutive
  // elements [tile * TE + t * EPV, ...) of every tile (coalesced 16-byte loads).
  // Each warp's sums per tile go to a shared table, in index order, so the
  // draw point's (tile, warp) is found by a scan of the table and that warp
  // alone re-reads its 32 * EPV elements to place it.
  const int pos = fin < 0 ? K : fin;
  const char* trow = tgt + static_cast<int64_t>(pos) * V * E::kSize;
  const char* drow = fin < 0 ? nullptr : drf + static_cast<int64_t>(fin) * V * E::kSize;
  const float smT = st[pos].smax;
  const double ZT = __ull2double_rn(st[pos].Z);
  const float smD = fin < 0 ? 0.0f : st[K + 1 + fin].smax;
  const double ZD = fin < 0 ? 1.0 : __ull2double_rn(st[K + 1 + fin].Z);
  const unsigned long long ZTi = __double2ull_rn(ZT), ZDi = __double2ull_rn(ZD);  // exact: integer values
  constexpr int EPV = E::kEPV;
  constexpr int NW = kSpecNT / 32;
  constexpr int TE = kSpecNT * EPV;
  const int lane = t & 31, warp = t >> 5;
  const int c0 = min(V, rank * a.chunk), c1 = min(V, c0 + a.chunk);
  const int n = c1 - c0;
  const int ntile = (n + TE - 1) / TE;
  extern __shared__ unsigned long long vtab[];  // [ntile * NW] target sums, then residual sums
  const uint32_t* msk = !kMask ? nullptr : spec_mask(a, b, pos);
  // c0 is a multiple of 8 elements: the slice starts on a 16-byte boundary
  // whenever the row does
  const bool vec = ((reinterpret_cast<uintptr_t>(trow) | reinterpret_cast<uintptr_t>(drow)) & 15u) == 0;
  // elements i0 .. i0 + EPV - 1 of the slice; -inf past its end or where masked
  auto load_epv = [&](const char* row, int i0, float* x) {
    if (vec && i0 + EPV <= n) {
      E::unpack(__ldg(reinterpret_cast<const uint4*>(row + static_cast<int64_t>(c0 + i0) * E::kSize)), x);
    } else {
#pragma unroll
      for (int e = 0; e < EPV; e++) x[e] = i0 + e < n ? E::load(row, c0 + i0 + e) : neg_inf();
    }
    if (msk) {
#pragma unroll
      for (int e = 0; e < EPV; e++)
        if (i0 + e < n && !mask_allows(msk, c0 + i0 + e)) x[e] = neg_inf();
    }
  };
  // every d = x / T - max(x / T) <= 0: the branch-free exact mass applies
  auto qmT = [&](float x) { return qmass_le0(__fsub_rn(__fdiv_rn(x, T), smT)); };
  auto qmD = [&](float x) { return qmass_le0(__fsub_rn(__fdiv_rn(x, T), smD)); };
  auto wsum = [&](unsigned long long w) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(kFull, w, o);
    return w;
  };
  unsigned long long sT = 0, sR = 0;
  for (int tile = 0; tile < ntile; tile++) {
    const int i0 = tile * TE + t * EPV;
    float xt[EPV];
    load_epv(trow, i0, xt);
    unsigned long long wt = 0, wr = 0;
    if (fin >= 0) {
      float xd[EPV];
      load_epv(drow, i0, xd);
#pragma unroll
      for (int e = 0; e < EPV; e++) {
        const unsigned long long qt = qmT(xt[e]);
        wt += qt;
        wr += resid_mass_x(qt, ZT, ZTi, qmD(xd[e]), ZD, ZDi);
      }
      wr = wsum(wr);
    } else {
#pragma unroll
      for (int e = 0; e < EPV; e++) wt += qmT(xt[e]);
    }
    wt = wsum(wt);
    sT += wt;
    sR += wr;
    if (lane == 0) {
      vtab[tile * NW + warp] = wt;
      vtab[(ntile + tile) * NW + warp] = wr;
    }
  }
  if (lane == 0) { sm.red_u64[warp] = sT; sm.red_u64[NW + warp] = sR; }
  __syncthreads();
  if (t == 0) {
    unsigned long long cT = 0, cR = 0;
    for (int w = 0; w < NW; w++) { cT += sm.red_u64[w]; cR += sm.red_u64[NW + w]; }
    c_sumT = cT;
    c_sumR = cR;
  }
  cluster.sync();
  unsigned long long totT = 0, totR = 0, preT = 0, preR = 0;
  for (int q = 0; q < kSpecCluster; q++) {
    const unsigned long long xT = *cluster.map_shared_rank(&c_sumT, q);
    const unsigned long long xR = *cluster.map_shared_rank(&c_sumR, q);
    if (q < rank) { preT += xT; preR += xR; }
    totT += xT;
    totR += xR;
  }
  const bool use_resid = fin >= 0 && __dmul_rn(__ull2double_rn(totR), 1.0 / kResidScale) > 1e-10;
  const unsigned long long total = use_resid ? totR : totT;
  const unsigned long long mine = use_resid ? *cluster.map_shared_rank(&c_sumR, rank) : *cluster.map_shared_rank(&c_sumT, rank);
  const unsigned long long before = use_resid ? preR : preT;
  const unsigned long long rpt = draw_point(a.u_draw[b], total);
  if (total == 0 && rank == 0 && t == 0) a.out_n[b] = n0;  // masked away entirely: no token
  if (mine > 0 && before <= rpt && rpt < before + mine) {  // CTA-uniform
    // the (tile, warp) entry holding the draw point, in index order
    const unsigned long long* tab = vtab + (use_resid ? ntile * NW : 0);
    if (t == 0) {
      unsigned long long c = before;
      int ent = ntile * NW - 1;
      for (int i = 0; i < ntile * NW; i++) {
        if (rpt < c + tab[i]) { ent = i; break; }
        c += tab[i];
      }
      s_ent = ent;
      s_before = c;
    }
    __syncthreads();
    const int ent = s_ent;
    if (warp == ent % NW) {
      const int i0 = (ent / NW) * TE + t * EPV;
      float xt[EPV], xd[EPV];
      unsigned long long q8[EPV], w = 0;
      load_epv(trow, i0, xt);
      if (use_resid) load_epv(drow, i0, xd);
#pragma unroll
      for (int e = 0; e < EPV; e++) {
        const unsigned long long qt = qmT(xt[e]);
        q8[e] = use_resid ? resid_mass_x(qt, ZT, ZTi, qmD(xd[e]), ZD, ZDi) : qt;
        w += q8[e];
      }
      unsigned long long incl = w;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long v = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += v;
      }
      const unsigned long long r2 = rpt - s_before;
      if (w > 0 && r2 >= incl - w && r2 < incl) {
        unsigned long long c = incl - w;
        int pick = c0 + i0 + EPV - 1;
#pragma unroll
        for (int e = 0; e < EPV; e++) {
          c += q8[e];
          if (c > r2) { pick = c0 + i0 + e; break; }
        }
        out[n0] = pick;
        a.out_n[b] = n0 + 1;
      }
    }
  }
  cluster.sync();  // keep this CTA's shared memory alive for its peers
}

// Launch on `st` as a programmatic dependent of the previous work on the
// stream (every spec kernel starts with griddepcontrol.wait), so each launch of
// the chain is set up while the previous one drains.  The cluster shape comes
// from the kernels' __cluster_dims__.
template <class... KArgs, class... Args>
inline cudaError_t spec_launch(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t st,
                               Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// One verification on `st`.  Eager: statistics of every position, then the
// chain and the draw (two launches).  Lazy (rstate given): statistics of
// position i only for the rows still accepting, i = 0..K-1, each followed by
// the accept test, then the bonus row of the rows that accepted everything,
// then the draw (2K + 2 launches, fewer vocab rows read).
template <int DT, bool kMask>
inline cudaError_t launch_spec_t(SpecArgs a, cudaStream_t st) {
  int chunk = (a.vocab + kSpecCluster - 1) / kSpecCluster;
  chunk = (chunk + 7) / 8 * 8;
  a.chunk = chunk;
  const size_t stage = 0;  // no dynamic shared memory
  cudaError_t e = cudaSuccess;
  if (!a.rstate) {
    const int nrows = a.batch * (2 * a.K + 1);
    e = spec_launch(spec_stats_kernel<DT, kMask>, nrows * kSpecCluster, kSpecNT, stage, st, a);
  } else {
    for (int i = 0; i < a.K && e == cudaSuccess; i++) {
      a.lazy_pos = i;
      e = spec_launch(spec_stats_kernel<DT, kMask>, a.batch * 2 * kSpecCluster, kSpecNT, stage, st, a);
      if (e == cudaSuccess)
        e = spec_launch(spec_chain_kernel<DT, kMask>, (a.batch + 127) / 128, 128, 0, st, a, i);
    }
    a.lazy_pos = a.K;
    if (e == cudaSuccess)
      e = spec_launch(spec_stats_kernel<DT, kMask>, a.batch * kSpecCluster, kSpecNT, stage, st, a);
  }
  // the verify kernel's table: two sums per (tile, warp) of a slice
  const int vtiles = (chunk + kSpecNT * Elt<DT>::kEPV - 1) / (kSpecNT * Elt<DT>::kEPV);
  const size_t vsmem = static_cast<size_t>(2 * vtiles * (kSpecNT / 32)) * sizeof(unsigned long long);
  if (e == cudaSuccess) e = spec_launch(spec_verify_kernel<DT, kMask>, a.batch * kSpecCluster, kSpecNT, vsmem, st, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// The masked kernels are separate instances, so the unmasked path carries no
// mask code.
template <int DT>
inline cudaError_t launch_spec(SpecArgs a, cudaStream_t st) {
  return a.state_ids ? launch_spec_t<DT, true>(a, st) : launch_spec_t<DT, false>(a, st);
}

}  // namespace tg
