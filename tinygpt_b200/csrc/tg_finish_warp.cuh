// tg_finish_warp.cuh -- the finishing half of the two-kernel mode, one warp per
// row.
//
// The streaming kernel leaves every row's candidate list (each element >= theta
// with its id) in global memory, where it stays L2-resident.  One warp per row
// stages that list once into a shared-memory pool and runs stages (a)
// penalties, (c) exact k-th value, (b) masses, (d) top-p / min-p and (e) the
// draw over it, with warp-synchronous histogram selections and no CTA-wide
// barrier; a CTA of up to 16 warps finishes that many rows at once, so a batch
// of 2048 rows finishes in one wave.  The arithmetic is the one finish_cands
// uses (tg_sample.cuh), so ids and probabilities are the same bit for bit.
//
// Reference semantics kept: python_ref/model.py:216-224 (greedy, /T, top-k with
// ties kept, softmax), wasm/src/model.cpp:508-516 (index-order inverse CDF),
// ModelController.swift:268-284 (repetition penalty on raw logits).
//
// Rows this finisher does not take are appended to a fallback list that the
// CTA-per-row kernel (sample_list_kernel over sample_row) finishes afterwards:
//   * rows the streaming kernel did not stream (cand_gn < 0: top-k > 1024,
//     bad grammar state, ...), rows without top-k, rows whose penalties can
//     raise a logit, histories longer than kWfMaxHist, rows the CTA's pool had
//     no room for;
//   * rows whose list holds fewer than k elements >= theta after the
//     penalties, or where an element below theta could tie the k-th tempered
//     value.
// The global lists are only read, so a row left for the fallback still has its
// raw list there.
#pragma once

#include "tg_sample.cuh"

namespace tg {

constexpr int kWfMaxWarps = 16;      // rows per CTA at most
#ifndef TG_WF_WARPS
#define TG_WF_WARPS 28
#endif
constexpr int kWfGroupWarps = TG_WF_WARPS;  // warps per CTA at most (65536 / (32 x this) registers per thread)
constexpr int kWfMaxNT = kWfGroupWarps * 32;
constexpr int kWfSmem = 227 * 1024 - 256;  // dynamic shared memory of a CTA (static: 64 B)
constexpr int kWfBins = 256;         // histogram bins of one selection round
constexpr int kWfMaxHist = 1024;     // longest history served (hash of 2048 slots)
constexpr int kWfBloomWords = 256;   // 8192-bit Bloom filter of the history ids

// A group of G warps that finishes one row.  G == 1 synchronizes with
// __syncwarp; larger groups with their own named barrier `bar` (1..15; 0 is
// __syncthreads').
template <int G>
struct Grp {
  static constexpr int NT = 32 * G;
  int id;    // group index in the CTA
  int gt;    // thread index in the group
  int gw;    // warp index in the group
  int lane;
  int bar;   // named barrier of the group (G > 1)
  __device__ __forceinline__ void sync() const {
    if constexpr (G == 1) {
      __syncwarp();
    } else {
      asm volatile("bar.sync %0, %1;" ::"r"(bar), "n"(NT) : "memory");
    }
  }
};

// Per-group selection scratch: bin weights, the small list of a crossing bin,
// and the group's reduction slots.
struct GrpSel {
  unsigned int hl[3][kWfBins];  // 15-bit limbs of the bin weights (masses <= 2^44)
  unsigned long long sk[32];
  unsigned long long sw[32];
  unsigned long long ru[4];     // per-warp partials
  unsigned long long rv[4];
  float rf[4];
  float rg[4];
  int ri[4];
  int cnt;
  int bin;
  unsigned long long bb;
  unsigned long long res_key;
  unsigned long long res_w;
  unsigned long long res_before;
  int res;                      // 0: not reached, 1: resolved, 2: narrow
};

// Per-group scratch: the Bloom filter, then the history hash (penalty pass
// only) sharing its bytes with the selection scratch.
__host__ __device__ __forceinline__ size_t grp_fin_bytes(int ht_log2) {
  const size_t h = ht_log2 ? (size_t(4) << ht_log2) : 0;
  const size_t s = sizeof(GrpSel);
  return 4 * kWfBloomWords + (((h > s ? h : s) + 15) & ~size_t(15));
}

// Warp-wide inclusive scan of u64.
__device__ __forceinline__ unsigned long long warp_incl_scan(unsigned long long v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long n = __shfl_up_sync(kFull, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Group sum of a u64 (every thread gets it).
template <int G>
__device__ __forceinline__ unsigned long long grp_sum(const Grp<G>& g, GrpSel& ws, unsigned long long v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  if constexpr (G == 1) return v;
  if (g.lane == 0) ws.ru[g.gw] = v;
  g.sync();
  unsigned long long r = 0;
#pragma unroll
  for (int i = 0; i < G; i++) r += ws.ru[i];
  g.sync();
  return r;
}

// Shift that maps key - lo, for keys in [lo, lo + width], onto 256 bins.
template <class K>
__device__ __forceinline__ int sel_shift(K width) {
  const int bits = sizeof(K) == 8 ? 64 - __clzll(static_cast<long long>(width))
                                  : 32 - __clz(static_cast<int>(width));
  return bits > 8 ? bits - 8 : 0;
}

template <bool kMass, int G>
__device__ __forceinline__ void sel_zero(const Grp<G>& g, GrpSel& ws) {
  for (int i = g.gt; i < kWfBins; i += 32 * G) {
    ws.hl[0][i] = 0u;
    if (kMass) { ws.hl[1][i] = 0u; ws.hl[2][i] = 0u; }
  }
}

template <bool kMass>
__device__ __forceinline__ void sel_put(GrpSel& ws, int bn, unsigned long long w) {
  if (kMass) {
    atomicAdd(&ws.hl[0][bn], static_cast<unsigned>(w & 0x7fffu));
    atomicAdd(&ws.hl[1][bn], static_cast<unsigned>((w >> 15) & 0x7fffu));
    atomicAdd(&ws.hl[2][bn], static_cast<unsigned>(w >> 30));
  } else {
    atomicAdd(&ws.hl[0][bn], 1u);
  }
}

// Weighted selection in ascending key order over the elements that iter(f)
// yields (f(key, value) per element, the group's threads striding; wt(key,
// value) gives the weight, 0 = not taking part; weights are counts when
// !kMass, else masses <= 2^44 summed in 15-bit limbs): the first element at
// which reached(weight of every element up to and including it) holds.
// Each round histograms the keys of [lo, hi] into 256 bins (bin = (key - lo) >>
// sh); warp 0 finds the crossing bin by a scan; then the bin is resolved
// exactly (<= 32 members, sorted in warp 0's registers; or all members share
// one key) or [lo, hi] narrows to the members' key range, at least 8 bits
// narrower.  With prefilled, the caller has already put the elements of round
// 0 into the histogram (sel_zero, then sel_put at bin (key - lo) >>
// sel_shift(hi - lo)) and synchronized the group.
// Outputs: the key, the weight strictly before it in key order, and its weight
// (when it is the only member with that key).  Returns false if reached() never
// holds (the caller falls back).
template <bool kMass, class K, int G, class Iter, class Wt, class Reached>
__device__ bool grp_select(const Grp<G>& g, Iter iter, Wt wt, K lo, K hi, bool prefilled, Reached reached,
                           GrpSel& ws, K& key_out, unsigned long long& before_out, unsigned long long& w_out) {
  const int lane = g.lane;
  unsigned long long before = 0;
  for (int round = 0; round <= 2 * static_cast<int>(sizeof(K)); round++) {
    const int sh = sel_shift<K>(hi - lo);
    if (!(prefilled && round == 0)) {
      sel_zero<kMass>(g, ws);
      g.sync();
      iter([&](K key, float v) {
        if (key < lo || key > hi) return;
        const unsigned long long w = wt(key, v);
        if (w) sel_put<kMass>(ws, static_cast<int>((key - lo) >> sh), w);
      });
      g.sync();
    }
    if (g.gw == 0) {  // warp 0: the crossing bin
      unsigned long long c[kWfBins / 32];
      unsigned long long loc = 0;
#pragma unroll
      for (int j = 0; j < kWfBins / 32; j++) {
        const int bn = lane * (kWfBins / 32) + j;
        c[j] = kMass ? static_cast<unsigned long long>(ws.hl[0][bn]) + (static_cast<unsigned long long>(ws.hl[1][bn]) << 15) +
                           (static_cast<unsigned long long>(ws.hl[2][bn]) << 30)
                     : static_cast<unsigned long long>(ws.hl[0][bn]);
        loc += c[j];
      }
      const unsigned long long incl = warp_incl_scan(loc);
      const unsigned bal = __ballot_sync(kFull, reached(before + incl));
      if (lane == 0) { ws.bin = -1; ws.cnt = 0; }
      __syncwarp();
      if (bal && lane == __ffs(bal) - 1) {
        unsigned long long cc = before + incl - loc;
#pragma unroll
        for (int j = 0; j < kWfBins / 32; j++) {
          if (reached(cc + c[j])) { ws.bin = lane * (kWfBins / 32) + j; ws.bb = cc; break; }
          cc += c[j];
        }
      }
    }
    g.sync();
    const int bin = ws.bin;
    const unsigned long long bb = ws.bb;
    if (bin < 0) return false;
    // members of the crossing bin: key range, count, the first 32
    const K blo = lo + (static_cast<K>(bin) << sh);
    const K span = (K(1) << sh) - K(1);
    const K bhi = hi - blo < span ? hi : blo + span;
    K kmin = ~K(0), kmax = K(0);
    iter([&](K key, float v) {
      if (key < blo || key > bhi) return;
      const unsigned long long w = wt(key, v);
      if (!w) return;
      kmin = key < kmin ? key : kmin;
      kmax = key > kmax ? key : kmax;
      const int pos = atomicAdd(&ws.cnt, 1);
      if (pos < 32) { ws.sk[pos] = static_cast<unsigned long long>(key); ws.sw[pos] = w; }
    });
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const K x = __shfl_xor_sync(kFull, kmin, o);
      const K y = __shfl_xor_sync(kFull, kmax, o);
      kmin = x < kmin ? x : kmin;
      kmax = y > kmax ? y : kmax;
    }
    if constexpr (G > 1) {
      if (lane == 0) { ws.ru[g.gw] = static_cast<unsigned long long>(kmin); ws.rv[g.gw] = static_cast<unsigned long long>(kmax); }
    }
    g.sync();
    if constexpr (G > 1) {
#pragma unroll
      for (int i = 0; i < G; i++) {
        const K x = static_cast<K>(ws.ru[i]), y = static_cast<K>(ws.rv[i]);
        kmin = x < kmin ? x : kmin;
        kmax = y > kmax ? y : kmax;
      }
    }
    const int n = ws.cnt;
    if (n == 0) return false;
    if (kmin == kmax) {  // one key: the crossing element has it
      w_out = n == 1 ? ws.sw[0] : 0ull;
      key_out = kmin;
      before_out = bb;
      g.sync();
      return true;
    }
    if (n <= 32) {  // warp 0 sorts the members by key and scans their weights
      if (g.gw == 0) {
        unsigned long long k = lane < n ? ws.sk[lane] : ~0ull;
        unsigned long long x = lane < n ? ws.sw[lane] : 0ull;
#pragma unroll
        for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
          for (int j = size >> 1; j > 0; j >>= 1) {
            const unsigned long long ok = __shfl_xor_sync(kFull, k, j);
            const unsigned long long ox = __shfl_xor_sync(kFull, x, j);
            const bool up = (lane & size) == 0;
            const bool lower = (lane & j) == 0;
            const bool take = (lower == up) ? (ok < k) : (ok > k);
            if (take) { k = ok; x = ox; }
          }
        }
        const unsigned long long inc = warp_incl_scan(x);
        const unsigned hit = __ballot_sync(kFull, lane < n && reached(bb + inc));
        if (lane == 0) ws.res = 0;
        __syncwarp();
        if (hit && lane == __ffs(hit) - 1) {
          ws.res = 1;
          ws.res_key = k;
          ws.res_w = x;
          ws.res_before = bb + inc - x;
        }
      }
      g.sync();
      const bool ok = ws.res == 1;
      key_out = static_cast<K>(ws.res_key);
      w_out = ws.res_w;
      before_out = ws.res_before;
      g.sync();
      return ok;
    }
    lo = kmin;
    hi = kmax;
    before = bb;
    g.sync();
  }
  return false;
}

// History hash slot: ((id + 1) << 11) | count; 0 = empty.  Counts stay below
// 2^11 because histories served here hold at most kWfMaxHist ids.
// Slot from the low bits of the mixed id hash (tg_mix32), Bloom bit from its
// high 13 bits.
__device__ __forceinline__ int wf_slot0(int id, int mask) {
  return static_cast<int>(tg_mix32(static_cast<uint32_t>(id))) & mask;
}
__device__ __forceinline__ uint32_t wf_bloom_bit(int id) {
  return tg_mix32(static_cast<uint32_t>(id)) >> 19;  // 13 bits
}

// Diagnostic build only (-DTG_PHASE_TIMING): cycles per stage of the warp
// finisher, summed over warps into g_phase_cycles[16 + i].
struct WarpClock {
  long long last = 0;
  __device__ __forceinline__ void mark(int i) {
#ifdef TG_PHASE_TIMING
    if ((threadIdx.x & 31) == 0) {
      const long long now = clock64();
      if (last) atomicAdd(&g_phase_cycles[16 + i], static_cast<unsigned long long>(now - last));
      last = now;
    }
#else
    (void)i;
#endif
  }
};

// The row's shared-memory pool entries (its list length) when this finisher
// takes the row, else 0.
__device__ __forceinline__ int warp_row_need(const SampleArgs& a, int b) {
  const int n = a.cand_gn[b];
  if (n <= 0 || n > kCandMax) return 0;
  const tg_row_params p = a.params[b];
  const bool greedy = !(p.temperature > 0.0f);
  const bool topk = p.top_k > 0 && p.top_k < a.vocab;
  return (greedy || topk) ? n : 0;
}

// Whether a finisher group takes row b, whose list holds n elements >= theta
// (n > kCandMax: the list overflowed).  Decided before the list is touched.
__device__ __forceinline__ bool grp_can_take(const SampleArgs& a, int b, int n, float theta) {
  if (n <= 0 || n > kCandMax || !(theta > neg_inf())) return false;
  const tg_row_params p = a.params[b];
  const bool greedy = !(p.temperature > 0.0f);
  const bool topk = p.top_k > 0 && p.top_k < a.vocab;
  if (!greedy && !topk) return false;
  int hlen = 0;
  if (a.history_len && a.history && a.hist_cap > 0) {
    hlen = a.history_len[b];
    hlen = hlen < 0 ? 0 : (hlen > a.hist_cap ? a.hist_cap : hlen);
  }
  const bool pf_on = p.presence_penalty != 0.0f || p.frequency_penalty != 0.0f;
  const bool need_hist = hlen > 0 && (p.repetition_penalty > 1.0f || pf_on);
  if (need_hist && pf_on && (p.presence_penalty < 0.0f || p.frequency_penalty < 0.0f)) return false;
  if (need_hist && hlen > kWfMaxHist) return false;
  return true;
}

// A group of G warps finishes row b (grp_can_take holds) over its list of n
// elements >= theta in ly / lid: staged there first from the global list when
// kFromGlobal, else already there (the fused kernel's slot).  The list is
// modified in place (penalties, compaction); the global list is only read.
// Returns false when the row is left for a fallback.
// Element i of the list belongs to warp (i / 32) % G; after the compaction each
// warp keeps its survivors in its own slots, in place (slot(j) below), so no
// cross-warp prefix is needed.
template <int G, bool kFromGlobal>
__device__ bool grp_finish_row(const Grp<G>& g, const SampleArgs& a, int b, int n, float theta,
                               unsigned char* scratch, float* ly, int* lid) {
  constexpr int NT = 32 * G;
  const int lane = g.lane, gt = g.gt;
  const tg_row_params p = a.params[b];
  const int V = a.vocab;
  const bool greedy = !(p.temperature > 0.0f);
  int hlen = 0;
  if (a.history_len && a.history && a.hist_cap > 0) {
    hlen = a.history_len[b];
    hlen = hlen < 0 ? 0 : (hlen > a.hist_cap ? a.hist_cap : hlen);
  }
  const bool rep_on = p.repetition_penalty > 1.0f;
  const bool pf_on = p.presence_penalty != 0.0f || p.frequency_penalty != 0.0f;
  const bool need_hist = hlen > 0 && (rep_on || pf_on);

  uint32_t* bloom = reinterpret_cast<uint32_t*>(scratch);
  uint32_t* hash = bloom + kWfBloomWords;
  GrpSel& ws = *reinterpret_cast<GrpSel*>(hash);
  WarpClock wc;
  wc.mark(0);
  const float* gy = a.cand_gy + static_cast<int64_t>(b) * kCandMax;
  const int* gid = a.cand_gid + static_cast<int64_t>(b) * kCandMax;

  // stage the list: 16 loads in flight per thread, straight to shared memory
  constexpr int LU = 16;
  for (int base = gt; kFromGlobal && base < n; base += NT * LU) {
    float yv[LU];
    int iv[LU];
#pragma unroll
    for (int q = 0; q < LU; q++) {
      const int i = base + NT * q;
      if (i < n) { yv[q] = __ldcg(gy + i); iv[q] = __ldcg(gid + i); }
    }
#pragma unroll
    for (int q = 0; q < LU; q++) {
      const int i = base + NT * q;
      if (i < n) { ly[i] = yv[q]; lid[i] = iv[q]; }
    }
  }

  // (a) history -> hash of distinct ids with counts, and a Bloom filter of them
  const int hmask = need_hist ? (1 << a.ht_log2) - 1 : 0;
  if (need_hist) {
    for (int i = gt; i <= hmask; i += NT) hash[i] = 0u;
    for (int i = gt; i < kWfBloomWords; i += NT) bloom[i] = 0u;
    g.sync();
    const int32_t* h = a.history + static_cast<int64_t>(b) * a.history_stride;
    constexpr int HU = 8;
    for (int base = gt; base < hlen; base += NT * HU) {
      int ids[HU];
#pragma unroll
      for (int q = 0; q < HU; q++) ids[q] = base + NT * q < hlen ? __ldg(h + base + NT * q) : -1;
#pragma unroll 1
      for (int q = 0; q < HU; q++) {
        int id = ids[0];
#pragma unroll
        for (int r = 1; r < HU; r++) id = q == r ? ids[r] : id;  // register select, no local memory
        if (id < 0 || id >= V) continue;
        const uint32_t tag = static_cast<uint32_t>(id + 1) << 11;
        int s = wf_slot0(id, hmask);
        for (;;) {
          const uint32_t old = atomicCAS(&hash[s], 0u, tag | 1u);
          if (old == 0u) {
            const uint32_t bit = wf_bloom_bit(id);
            atomicOr(&bloom[bit >> 5], 1u << (bit & 31));
            break;
          }
          if ((old & ~0x7ffu) == tag) { atomicAdd(&hash[s], 1u); break; }
          s = (s + 1) & hmask;
        }
      }
    }
  }
  g.sync();
  wc.mark(0);  // 16: staging and hash build
  if (a.debug_stop == 1) return false;
  auto count_of = [&](int id) {
    const uint32_t bit = wf_bloom_bit(id);
    if (!((bloom[bit >> 5] >> (bit & 31)) & 1u)) return 0;
    const uint32_t tag = static_cast<uint32_t>(id + 1) << 11;
    int s = wf_slot0(id, hmask);
    for (;;) {
      const uint32_t v = hash[s];
      if (v == 0u) return 0;
      if ((v & ~0x7ffu) == tag) return static_cast<int>(v & 0x7ffu);
      s = (s + 1) & hmask;
    }
  };

  // penalties in place; count, range and first argmax of the elements >= theta
  unsigned int cnt = 0;
  float ymax = neg_inf(), nymin = neg_inf();
  int amax = 0x7fffffff;
#pragma unroll 2
  for (int i = gt; i < n; i += NT) {
    float y = ly[i];
    const int id = lid[i];
    if (need_hist) {
      const int c = count_of(id);
      if (c > 0) {
        if (y != neg_inf()) {
          if (rep_on) y = y > 0.0f ? __fdiv_rn(y, p.repetition_penalty) : __fmul_rn(y, p.repetition_penalty);
          if (pf_on)
            y = __fsub_rn(y, __fadd_rn(__fmul_rn(p.frequency_penalty, static_cast<float>(c)), p.presence_penalty));
        }
        ly[i] = y;
      }
    }
    if (y >= theta) {
      cnt++;
      if (y > ymax || (y == ymax && id < amax)) { ymax = y; amax = id; }
      nymin = fmaxf(nymin, -y);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    cnt += __shfl_xor_sync(kFull, cnt, o);
    const float oy = __shfl_xor_sync(kFull, ymax, o);
    const int oi = __shfl_xor_sync(kFull, amax, o);
    if (oy > ymax || (oy == ymax && oi < amax)) { ymax = oy; amax = oi; }
    nymin = fmaxf(nymin, __shfl_xor_sync(kFull, nymin, o));
  }
  g.sync();  // the hash is dead from here; its bytes become ws
  if constexpr (G > 1) {
    if (lane == 0) { ws.ru[g.gw] = cnt; ws.rf[g.gw] = ymax; ws.ri[g.gw] = amax; ws.rg[g.gw] = nymin; }
    g.sync();
    cnt = 0;
    ymax = neg_inf();
    nymin = neg_inf();
    amax = 0x7fffffff;
#pragma unroll
    for (int w = 0; w < G; w++) {
      cnt += static_cast<unsigned int>(ws.ru[w]);
      const float oy = ws.rf[w];
      const int oi = ws.ri[w];
      if (oy > ymax || (oy == ymax && oi < amax)) { ymax = oy; amax = oi; }
      nymin = fmaxf(nymin, ws.rg[w]);
    }
    g.sync();
  }
  wc.mark(1);  // 17: penalty pass
  if (a.debug_stop == 2) return false;

  const unsigned int need = greedy ? 1u : static_cast<unsigned int>(p.top_k);
  if (cnt < need) return false;
  if (greedy) {
    if (gt == 0) {
      a.out_ids[b] = amax;
      if (a.out_probs) a.out_probs[b] = 1.0f;
    }
    return true;
  }
  const float T = p.temperature;

  // (c) exact k-th largest value over the elements >= theta (ties kept)
  uint32_t kk;
  unsigned long long kb, kw;
  const unsigned int k = static_cast<unsigned int>(p.top_k);
  const bool okk = grp_select<false, uint32_t>(
      g,
      [&](auto&& f) {
#pragma unroll 2
        for (int i = gt; i < n; i += NT) {
          const float y = ly[i];
          if (y >= theta) f(~fkey(y), y);
        }
      },
      [](uint32_t, float) { return 1ull; }, ~fkey(ymax), ~fkey(-nymin), false,
      [&](unsigned long long c) { return c >= k; }, ws, kk, kb, kw);
  if (!okk) return false;
  wc.mark(2);  // 18: k-th value
  if (a.debug_stop == 3) return false;
  const float kth = key2f(~kk);
  const float sk = __fdiv_rn(kth, T);
  const float below = key2f(fkey(theta) - 1u);  // every absent value is <= below
  if (__fdiv_rn(below, T) >= sk) return false;

  // (b) survivors compacted in place (tempered value, id) per warp, their
  // mass total, and the first top-p histogram round over their (s desc, id
  // asc) keys
  const float smax = __fdiv_rn(ymax, T);
  // every value below kth has a quotient below sk when the next float down does
  // (__fdiv_rn is monotone in y)
  const bool below_kth_out = __fdiv_rn(key2f(fkey(kth) - 1u), T) < sk;
  const bool toppon = p.top_p < 1.0f;
  const unsigned long long plo = static_cast<unsigned long long>(~fkey(smax)) << 32;
  const unsigned long long phi = (static_cast<unsigned long long>(~fkey(sk)) << 32) | 0xffffffffull;
  const int psh = sel_shift<unsigned long long>(phi - plo);
  auto pkey = [](float sv, int id) {
    return (static_cast<unsigned long long>(~fkey(sv)) << 32) | static_cast<uint32_t>(id);
  };
  if (toppon) sel_zero<true>(g, ws);
  g.sync();
  auto slot = [&](int j) { return (j >> 5) * NT + g.gw * 32 + (j & 31); };
  const unsigned lt = (1u << lane) - 1u;
  int m = 0;  // this warp's survivors
  unsigned long long Q = 0;
#pragma unroll 1
  for (int base = 0; base < n; base += NT) {
    const int i = base + g.gw * 32 + lane;
    const float y = i < n ? ly[i] : neg_inf();
    const int id = i < n ? lid[i] : -1;
    __syncwarp();  // writes go only to this warp's slots at or below those loaded
    float sv = 0.0f;
    // y >= kth keeps (division is monotone); below kth only a value whose
    // quotient can still round up to sk needs the division
    bool keep = y >= theta && y > neg_inf() && (y >= kth || !below_kth_out);
    if (keep) {
      sv = __fdiv_rn(y, T);
      keep = sv >= sk;
    }
    if (keep) {
      const unsigned long long q = qmass_le0(__fsub_rn(sv, smax));
      Q += q;
      if (toppon && q) sel_put<true>(ws, static_cast<int>((pkey(sv, id) - plo) >> psh), q);
    }
    const unsigned bal = __ballot_sync(kFull, keep);
    if (keep) {
      const int pos = slot(m + __popc(bal & lt));
      ly[pos] = sv;
      lid[pos] = id;
    }
    m += __popc(bal);
  }
  __syncwarp();
  Q = grp_sum(g, ws, Q);  // its barriers also publish the top-p histogram
  wc.mark(3);  // 19: compaction and Q
  if (a.debug_stop == 4) return false;

  auto mass = [&](float sv) { return qmass_le0(__fsub_rn(sv, smax)); };
  // (d) top-p: the last element (cut_key, cut_id) of the shortest prefix in
  // (s desc, id asc) order whose mass reaches top_p * Q
  uint32_t cut_key = 0;
  int cut_id = 0x7fffffff;
  if (toppon) {
    const double tau = __dmul_rn(static_cast<double>(p.top_p), __ull2double_rn(Q));
    if (tau > 0.0) {
      unsigned long long ck, cb, cw;
      const bool ok = grp_select<true, unsigned long long>(
          g,
          [&](auto&& f) {
#pragma unroll 2
            for (int j = lane; j < m; j += 32) {
              const int i = slot(j);
              const float sv = ly[i];
              f(pkey(sv, lid[i]), sv);
            }
          },
          [&](unsigned long long, float sv) { return mass(sv); }, plo, phi, true,
          [&](unsigned long long c) { return __ull2double_rn(c) >= tau; }, ws, ck, cb, cw);
      if (!ok) return false;
      cut_key = ~static_cast<uint32_t>(ck >> 32);
      cut_id = static_cast<int>(static_cast<uint32_t>(ck));
    } else {  // top_p <= 0: the single top element (smallest id among the maxima)
      cut_key = fkey(smax);
      unsigned long long best = 0;  // max of ~id
      for (int j = lane; j < m; j += 32) {
        const int i = slot(j);
        if (fkey(ly[i]) == cut_key) best = max(best, static_cast<unsigned long long>(~static_cast<uint32_t>(lid[i])));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(kFull, best, o));
      if constexpr (G > 1) {
        if (lane == 0) ws.ru[g.gw] = best;
        g.sync();
#pragma unroll
        for (int w = 0; w < G; w++) best = max(best, ws.ru[w]);
        g.sync();
      }
      cut_id = static_cast<int>(~static_cast<uint32_t>(best));
    }
  }
  wc.mark(4);  // 20: top-p
  if (a.debug_stop == 5) return false;
  const bool minpon = p.min_p > 0.0f;
  const double minq = __dmul_rn(static_cast<double>(fminf(p.min_p, 1.0f)), static_cast<double>(kMassScale));
  auto kept_mass = [&](float sv, int id) {
    const unsigned long long q = mass(sv);
    if (toppon) {
      const uint32_t kq = fkey(sv);
      if (!(kq > cut_key || (kq == cut_key && id <= cut_id))) return 0ull;
    }
    if (minpon && !(__ull2double_rn(q) >= minq)) return 0ull;
    return q;
  };
  // kept mass S, and the first draw histogram round over ids
  const int dsh = sel_shift<uint32_t>(static_cast<uint32_t>(V - 1));
  sel_zero<true>(g, ws);
  g.sync();
  unsigned long long S = 0;
#pragma unroll 2
  for (int j = lane; j < m; j += 32) {
    const int i = slot(j);
    const int id = lid[i];
    const unsigned long long q = kept_mass(ly[i], id);
    S += q;
    if (q) sel_put<true>(ws, id >> dsh, q);
  }
  S = grp_sum(g, ws, S);
  if (S == 0) return false;
  wc.mark(5);  // 21: kept mass S
  if (a.debug_stop == 6) return false;

  // (e) draw: the first id in index order whose running mass exceeds r
  const unsigned long long r = draw_point(a.uniforms ? a.uniforms[b] : 0.0f, S);
  uint32_t pk;
  unsigned long long pb, pw;
  const bool okd = grp_select<true, uint32_t>(
      g,
      [&](auto&& f) {
#pragma unroll 2
        for (int j = lane; j < m; j += 32) {
          const int i = slot(j);
          f(static_cast<uint32_t>(lid[i]), ly[i]);
        }
      },
      [&](uint32_t id, float sv) { return kept_mass(sv, static_cast<int>(id)); }, 0u,
      static_cast<uint32_t>(V - 1), true, [&](unsigned long long c) { return c > r; }, ws, pk, pb, pw);
  if (!okd) return false;
  wc.mark(6);  // 22: draw
  if (a.debug_stop == 7) return false;
  if (gt == 0) {
    a.out_ids[b] = static_cast<int>(pk);
    if (a.out_probs) a.out_probs[b] = __double2float_rn(__ddiv_rn(__ull2double_rn(pw), __ull2double_rn(S)));
  }
  return true;
}

// One CTA per SM, one group of G warps per row (blockDim.x / (32 G) rows per
// CTA).  The dynamic shared memory holds each group's scratch, then a pool that
// the CTA's rows share for their staged lists (a row beyond the pool goes to
// the fallback list).  Rows a group does not finish go to the fallback list.
template <int G>
__global__ void __launch_bounds__(kWfMaxNT, 1) finish_warp_kernel(SampleArgs a, int pool_entries) {
  // launched as a programmatic dependent of the streaming kernel: its lists are
  // complete and visible once this returns (a no-op for an ordinary launch)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ int needs[kWfMaxWarps];
  const int R = blockDim.x / (32 * G);  // rows of this CTA
  const Grp<G> g{static_cast<int>(threadIdx.x) / (32 * G), static_cast<int>(threadIdx.x) % (32 * G),
                 (static_cast<int>(threadIdx.x) % (32 * G)) >> 5, static_cast<int>(threadIdx.x) & 31,
                 static_cast<int>(threadIdx.x) / (32 * G) + 1};
  const int b = blockIdx.x * R + g.id;
  if (g.gt == 0) needs[g.id] = b < a.batch ? warp_row_need(a, b) : 0;
  __syncthreads();
  if (b >= a.batch) return;
  int off = 0;
  for (int v = 0; v < g.id; v++) off += needs[v];
  const int need = needs[g.id];
  const size_t wsb = grp_fin_bytes(a.ht_log2);
  float* py = reinterpret_cast<float*>(dyn + static_cast<size_t>(R) * wsb);
  int* pi = reinterpret_cast<int*>(py + pool_entries);
  const bool fits = need > 0 && off + need <= pool_entries;
  const int n = a.cand_gn[b];
  const float theta = a.cand_gth[b];
  const bool ok = fits && grp_can_take(a, b, n, theta) &&
                  grp_finish_row<G, true>(g, a, b, n, theta, dyn + static_cast<size_t>(g.id) * wsb, py + off, pi + off);
  if (g.gt == 0) {
    if (ok) {
      atomicAdd(&a.counters[0], 1ull);
      atomicAdd(&a.counters[6], 1ull);
    } else {
      if (!fits && need > 0) atomicAdd(&a.counters[7], 1ull);  // pool full
      const int pos = atomicAdd(a.fb_count, 1);
      a.fb_rows[pos] = b;
    }
  }
}

}  // namespace tg
