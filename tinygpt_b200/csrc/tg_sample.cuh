// tg_sample.cuh -- the fused sampling kernel: penalties + grammar mask +
// temperature + top-k + top-p / min-p + inverse-CDF draw, one CTA per row.
//
// Reference path (sarthak-fleet/tinygpt): python_ref/model.py:213-224,
// wasm/src/model.cpp:489-517, ModelController.swift:262-304,
// ConstrainedGen.swift:775-837, Serve.swift:1483-1506.
//
// Structure of one row (one CTA):
//   (a) penalty-and-mask: history ids go into a shared-memory hash (id -> count
//       -> penalised value); the mask row is gathered by state id and applied
//       to every 128-bit vector as it streams in.
//   (c) top-k prefilter: a sample of the row (the first vectors of every
//       thread) gives a threshold theta expected to pass ~1.5k+64 elements;
//       the single HBM pass appends every element >= theta to a shared-memory
//       candidate list (warp-aggregated, ballot-based).  The pass is one
//       128-bit load plus a vector max and a compare per 16 bytes.
//       The exact k-th value is then a radix select over the candidates.  If
//       the list overflowed or holds fewer than k elements >= theta, the row
//       is redone by the full-row path below (same stages, over global memory).
//   (b) softmax as exact fixed-point masses q = trunc(tg_exp(s - max) * 2^44).
//   (d) top-p: a mass-weighted radix search in (s desc, id asc) order; min-p:
//       a threshold on q.
//   (e) draw: r = trunc(u * S); a mass-weighted radix search over ids in
//       ascending order finds the first id whose running mass exceeds r.
#pragma once

#include "../../include/tgsample.h"
#include "tg_block.cuh"

namespace tg {

#ifndef TG_CAND_MAX
#define TG_CAND_MAX 2816
#endif
constexpr int kSampleNT = 256;         // threads per CTA (the default; kernels take NT)
constexpr int kCandMax = TG_CAND_MAX;   // candidate list capacity
constexpr int kFastMaxK = 1024;  // largest top-k served by the candidate path
constexpr int kSampleVecs = 4;   // 128-bit vectors per thread in the threshold sample
#ifndef TG_UNROLL
#define TG_UNROLL 4
#endif
constexpr int kUnroll = TG_UNROLL;  // 128-bit loads in flight per thread
constexpr int kNoTopkTarget = 512;  // candidate target of rows without top-k
// ... in the streaming kernel and the 256-thread CTA-per-row kernels: a longer
// list holds the top-p cut more often, so fewer rows fail their list and
// re-stream (config-4 rows without top-k 2822 -> 2523 us with the stream alone);
// the 1024-thread kernel of small batches keeps 512 (config 2 took 49 -> 144 us
// with 1024)
constexpr int kNoTopkTargetStream = 1024;
constexpr int kRetries = 2;      // threshold retries (re-streamed from L2) before the full row
#ifndef TG_MIN_CTAS
#define TG_MIN_CTAS 4
#endif
constexpr int kMinCtasPerSm = TG_MIN_CTAS;  // occupancy target (4: registers capped at 64)
#ifndef TG_STREAM_CTAS
#define TG_STREAM_CTAS 5
#endif
constexpr int kStreamCtasPerSm = TG_STREAM_CTAS;  // occupancy of the streaming kernel
// Candidate target of the threshold: the sample estimates the element of rank
// kTgtMul * k + kTgtAdd; the margin over k absorbs the sample's error (tighter
// margins measured slower: more rows needed a second pass).
#ifndef TG_TGT_MUL
#define TG_TGT_MUL 1.5f
#endif
#ifndef TG_TGT_ADD
#define TG_TGT_ADD 96.0f
#endif
constexpr float kTgtMul = TG_TGT_MUL;
constexpr float kTgtAdd = TG_TGT_ADD;
constexpr int kRing = 64;  // hit-vector ring entries per warp (drained at 32)
// the streaming kernel's rings take up to a whole 4-vector warp group (128
// entries) on top of fewer than 32 left over
constexpr int kStreamRing = 160;
static_assert((kSampleNT / 32) * kRing * 20 <= kCandMax * 4, "rings must fit in cand_e");
constexpr int kWideNT = 1024;  // threads per CTA for small batches
// Batches of kWideMinBatch..kWideMaxBatch rows run on wide CTAs (measured: a
// 1024-thread CTA makes 64 rows without top-k 2.3x faster; a single top-k row is
// faster on 256 threads).
constexpr int kWideMinBatch = 8;
constexpr int kWideMaxBatch = 148;
static_assert(kCandMax <= kWideMassN, "candidate mass histograms must not overflow their limbs");

// Diagnostic build only (-DTG_PHASE_TIMING): cycles per phase summed over CTAs.
#ifdef TG_PHASE_TIMING
__device__ unsigned long long g_phase_cycles[32];
// cycles per phase of rows 0..255 (16 phases each), summed over calls
__device__ unsigned long long g_row_phase[256 * 16];
#endif
struct PhaseClock {
  long long last = 0;
  int row = -1;
  __device__ __forceinline__ void mark(int i) {
#ifdef TG_PHASE_TIMING
    if (threadIdx.x == 0) {
      const long long now = clock64();
      if (last) {
        atomicAdd(&g_phase_cycles[i], static_cast<unsigned long long>(now - last));
        if (row >= 0 && row < 256 && i < 16) atomicAdd(&g_row_phase[row * 16 + i], static_cast<unsigned long long>(now - last));
      }
      last = now;
    }
#else
    (void)i;
#endif
  }
};

struct SampleArgs {
  const void* logits;
  int64_t row_stride;
  int32_t vocab;
  int32_t batch;
  const tg_row_params* params;
  const int32_t* history;
  const int32_t* history_len;
  int32_t history_stride;
  int32_t hist_cap;   // min(history_stride, TG_MAX_HISTORY), 0 if no history
  int32_t ht_log2;    // log2 of the hash size (0 if no history)
  const uint32_t* mask_table;
  int32_t num_states;
  int32_t mask_words;
  const int32_t* state_id;
  const float* uniforms;
  int32_t* out_ids;
  float* out_probs;
  uint32_t* status;
  unsigned long long* counters;  // TG_PATH_* counters
  // vocab-sharded mode: this call sees ids [vocab_offset, vocab_offset + vocab)
  // of rows of full_vocab ids and writes one record per row instead of ids
  int32_t vocab_offset;
  int32_t full_vocab;
  tg_shard_record* shard_out;
  // two-kernel mode: the streaming kernel leaves each row's raw candidate list
  // (every element >= theta, kCandMax slots per row), its length (-1: row not
  // streamed) and theta here; the finishing kernel starts from them
  float* cand_gy;
  int32_t* cand_gid;
  int32_t* cand_gn;
  float* cand_gth;
  // warp finisher: rows it left for sample_list_kernel, and their count
  int32_t* fb_rows;
  int32_t* fb_count;
  int32_t debug_stop;  // diagnostics: the warp finisher leaves rows after this stage (0: off)
  // streaming kernel: theta of every row is already in cand_gth (theta_kernel)
  int32_t theta_given;
};

// History hash in shared memory: key = token id (-1 empty); val = count, then
// the penalised value's float bits.  A 4096-bit Bloom word set filters lookups.
struct Hist {
  int* key;
  int* val;
  uint32_t* bloom;
  int mask;
  int log2;
  int active;
  // Bloom bit (12 bits) from the low bits of the same mixed hash, the slot
  // from its high bits
  __device__ __forceinline__ static uint32_t bloom_bit(int id) { return tg_mix32(static_cast<uint32_t>(id)) & 4095u; }
  __device__ __forceinline__ int slot0(int id) const {
    return static_cast<int>(tg_mix32(static_cast<uint32_t>(id)) >> (32 - log2));  // high bits
  }
  __device__ __forceinline__ bool find(int id, float& y) const {
    if (!active) return false;
    const uint32_t h = bloom_bit(id);
    if (!((bloom[h >> 5] >> (h & 31)) & 1u)) return false;
    int s = slot0(id);
    for (;;) {
      const int k = key[s];
      if (k == id) { y = __int_as_float(val[s]); return true; }
      if (k == -1) return false;
      s = (s + 1) & mask;
    }
  }
};

// Every element of the row, recomputed from global memory (L2 after the first
// pass): 128-bit loads over the aligned middle, scalars for head and tail.
template <int DT, int NT = kSampleNT>
struct GlobalSrc {
  const char* row;
  int V, head, nvec, tail0;
  const uint32_t* mask;
  Hist hist;
  int moff;  // bit offset of element 0 in the mask row (vocab shards)
  // value of element v (raw x): penalised, or -inf where masked
  __device__ __forceinline__ float value(int v, float x) const {
    float y;
    if (!hist.find(v, y)) y = (mask && !mask_allows(mask, v + moff)) ? neg_inf() : x;
    return y;
  }
  // values of vector j (elements head + j*EPV ...)
  __device__ __forceinline__ void vec(int j, float* y) const {
    using E = Elt<DT>;
    constexpr int EPV = E::kEPV;
    float x[EPV];
    E::unpack(__ldg(reinterpret_cast<const uint4*>(row + head * E::kSize) + j), x);
    const int e0 = head + j * EPV;
    const uint32_t bits = mask ? mask_bits(mask, e0 + moff, EPV) : 0xffu;
#pragma unroll
    for (int e = 0; e < EPV; e++)
      if (!hist.find(e0 + e, y[e])) y[e] = ((bits >> e) & 1u) ? x[e] : neg_inf();
  }
  template <class F>
  __device__ __forceinline__ void for_each(F&& f) const {
    using E = Elt<DT>;
    constexpr int EPV = E::kEPV;
    auto one = [&](int v, float x) {
      float y;
      if (!hist.find(v, y)) y = (mask && !mask_allows(mask, v + moff)) ? neg_inf() : x;
      f(v, y);
    };
    const int t = threadIdx.x;
    if (t < head) one(t, E::load(row, t));
    if (t < V - tail0) one(tail0 + t, E::load(row, tail0 + t));
    const uint4* vrow = reinterpret_cast<const uint4*>(row + head * E::kSize);
    for (int j = t; j < nvec; j += NT) {
      float x[EPV];
      E::unpack(__ldg(vrow + j), x);
      const int e0 = head + j * EPV;
      const uint32_t bits = mask ? mask_bits(mask, e0 + moff, EPV) : 0xffu;
#pragma unroll
      for (int e = 0; e < EPV; e++) {
        float y;
        if (!hist.find(e0 + e, y)) y = ((bits >> e) & 1u) ? x[e] : neg_inf();
        f(e0 + e, y);
      }
    }
  }
};

template <int NT = kSampleNT>
struct SmemSrcT {
  const float* y;
  const int* id;
  int n;
  float theta;
  template <class F>
  __device__ __forceinline__ void for_each(F&& f) const {
    for (int i = threadIdx.x; i < n; i += NT) {
      const float v = y[i];
      const int d = id[i];
      if (d >= 0 && v >= theta) f(d, v);
    }
  }
};

template <int N>
struct RegSrc {  // N values per thread, held in registers
  const float* v;
  template <class F>
  __device__ __forceinline__ void for_each(F&& f) const {
#pragma unroll
    for (int i = 0; i < N; i++) f(threadIdx.x, v[i]);
  }
};

template <int NT = kSampleNT, class Src>
__device__ __forceinline__ unsigned int block_count_if(const Src& src, float thr, BlockScratch& sm) {
  unsigned long long c = 0;
  src.for_each([&](int, float y) { c += (y >= thr) ? 1ull : 0ull; });
  return static_cast<unsigned int>(block_sum<NT>(c, sm));
}

// Stages (b)-(e) over a source.  Returns false (and writes nothing) when the
// source is a candidate list that turns out to miss an element the top-k
// threshold keeps; the caller then reruns the row over the full row.
template <int NT = kSampleNT, class Src>
__device__ bool finish_row(const Src& src, const tg_row_params& p, int V, float u,
                           bool check_theta, float theta, BlockScratch& sm, int& out_id,
                           float& out_prob) {
  if (!(p.temperature > 0.0f)) {  // greedy: first index of the maximum
    float y = neg_inf();
    int id = 0x7fffffff;
    src.for_each([&](int i, float v) {
      if (v > y || (v == y && i < id)) { y = v; id = i; }
    });
    block_argmax<NT>(y, id, sm);
    if (y == neg_inf()) { out_id = -1; out_prob = 0.0f; }
    else { out_id = id; out_prob = 1.0f; }
    return true;
  }
  const float T = p.temperature;
  const bool topk = p.top_k > 0 && p.top_k < V;
  float sk = neg_inf();
  if (topk) {
    uint32_t kkey; unsigned long long b0, m0; unsigned int c0, n0;
    const unsigned int k = static_cast<unsigned int>(p.top_k);
    radix_find<NT, true, false>(
        src, 32,
        [&](int, float y, uint32_t& key, unsigned long long& w) { key = fkey(y); w = 0; return true; },
        [&](unsigned long long, unsigned int c) { return c >= k; }, sm, kkey, b0, c0, n0, m0);
    const float kth = key2f(kkey);
    sk = __fdiv_rn(kth, T);
    if (check_theta && theta > neg_inf()) {
      // every element below theta is absent; none of them may reach sk
      const float bk = key2f(fkey(theta) - 1u);  // next float below theta
      if (__fdiv_rn(bk, T) >= sk) return false;
    }
  }
  float ymax = neg_inf();
  src.for_each([&](int, float y) { ymax = fmaxf(ymax, y); });
  ymax = block_max<NT>(ymax, sm);
  if (ymax == neg_inf()) { out_id = -1; out_prob = 0.0f; return true; }
  const float smax = __fdiv_rn(ymax, T);
  // y <= ylim implies y/T - smax <= -31.9, a zero mass (tg_exp(-31) * 2^44 < 1):
  // the rounding of ylim, y/T and the difference stays below 0.1 while
  // |smax| < 1e5.  Zero-mass elements change no sum, cut or draw, so their
  // division and exponential are skipped.
  const float ylim = __fmul_rn(__fsub_rn(smax, 32.0f), T);
  const bool use_lim = fabsf(smax) < 1.0e5f;
  auto mass = [&](float y, float s) {
    return (use_lim && !(y > ylim)) ? 0ull : qmass_le0(__fsub_rn(s, smax));
  };

  auto inA = [&](float y, float& s) {
    if (!(y > neg_inf())) return false;
    s = __fdiv_rn(y, T);
    return !topk || s >= sk;
  };

  unsigned long long Q = 0;
  src.for_each([&](int, float y) {
    if (!topk && use_lim && !(y > ylim)) return;  // zero mass
    float s;
    if (inA(y, s)) Q += mass(y, s);
  });
  Q = block_sum<NT>(Q, sm);

  // (d) top-p: last element (cut_key, cut_id) of the shortest (s desc, id asc)
  // prefix whose mass reaches top_p * Q.
  const bool toppon = p.top_p < 1.0f;
  uint32_t cut_key = 0;
  int cut_id = 0x7fffffff;
  if (toppon) {
    const double tau = __dmul_rn(static_cast<double>(p.top_p), __ull2double_rn(Q));
    unsigned long long above = 0, qt = 0;
    unsigned int nties = 0;
    unsigned long long jstar = 1;
    if (!(tau > 0.0)) {
      cut_key = fkey(smax);
      unsigned long long c = 0;
      src.for_each([&](int, float y) {
        float s;
        if (inA(y, s) && fkey(s) == cut_key) c++;
      });
      nties = static_cast<unsigned int>(block_sum<NT>(c, sm));
    } else {
      unsigned int cb;
      radix_find<NT, true, true>(
          src, 32,
          [&](int, float y, uint32_t& key, unsigned long long& w) {
            float s;
            if (!inA(y, s)) return false;
            key = fkey(s);
            w = mass(y, s);
            return true;
          },
          [&](unsigned long long m, unsigned int) { return __ull2double_rn(m) >= tau; }, sm,
          cut_key, above, cb, nties, qt);
      qt = qmass(__fsub_rn(key2f(cut_key), smax));
      if (qt > 0) {
        const double need = tau - __ull2double_rn(above);
        if (need > 0.0) {
          const double est = ceil(__ddiv_rn(need, __ull2double_rn(qt)));
          jstar = est < 1.0 ? 1ull : static_cast<unsigned long long>(est);
        }
        if (jstar > nties) jstar = nties;
        while (jstar > 1 && __ull2double_rn(above + (jstar - 1) * qt) >= tau) jstar--;
        while (jstar < nties && __ull2double_rn(above + jstar * qt) < tau) jstar++;
      }
    }
    if (jstar < nties) {
      uint32_t idkey; unsigned long long b1, m1; unsigned int c1, n1;
      const unsigned int js = static_cast<unsigned int>(jstar);
      radix_find<NT, false, false>(
          src, 20,
          [&](int id, float y, uint32_t& key, unsigned long long& w) {
            float s;
            if (!inA(y, s) || fkey(s) != cut_key) return false;
            key = static_cast<uint32_t>(id);
            w = 0;
            return true;
          },
          [&](unsigned long long, unsigned int c) { return c >= js; }, sm, idkey, b1, c1, n1, m1);
      cut_id = static_cast<int>(idkey);
    }
  }
  const bool minpon = p.min_p > 0.0f;
  const double minq = __dmul_rn(static_cast<double>(fminf(p.min_p, 1.0f)),
                                static_cast<double>(kMassScale));
  auto inF = [&](int id, float y, unsigned long long& q) {
    float s;
    if (!inA(y, s)) return false;
    if (toppon) {
      const uint32_t k = fkey(s);
      if (k < cut_key || (k == cut_key && id > cut_id)) return false;
    }
    q = mass(y, s);
    return !minpon || __ull2double_rn(q) >= minq;
  };

  unsigned long long S = 0;
  src.for_each([&](int id, float y) {
    unsigned long long q;
    if (inF(id, y, q)) S += q;
  });
  S = block_sum<NT>(S, sm);
  const unsigned long long r = draw_point(u, S);

  uint32_t pick; unsigned long long b2, qpick; unsigned int c2, n2;
  radix_find<NT, false, true>(
      src, 20,
      [&](int id, float y, uint32_t& key, unsigned long long& w) {
        if (!inF(id, y, w)) return false;
        key = static_cast<uint32_t>(id);
        return true;
      },
      [&](unsigned long long m, unsigned int) { return m > r; }, sm, pick, b2, c2, n2, qpick);
  out_id = static_cast<int>(pick);
  out_prob = __double2float_rn(__ddiv_rn(__ull2double_rn(qpick), __ull2double_rn(S)));
  return true;
}

// Full-row stages for a stochastic row without top-k (top-p, min-p or neither),
// in four passes over the row:
//   1. the maximum;
//   2. (top-p) the masses into a 1024-bin histogram over smax - s (32 bins per
//      unit, 32-bit limb atomics) and their total Q; the bin where the mass in
//      (s desc) order reaches top_p * Q is collected into shared memory and the
//      cut (key, id) resolved there exactly;
//   3. the final masses (top-p cut, min-p), summed per 128-bit-vector iteration
//      into a shared table (index order is iteration-major), and their total S;
//   4. the draw point's iteration recomputed: a block scan over its vectors and
//      one thread's scan of its own vector give the id.
// Same arithmetic as finish_row; returns false (nothing written) when the
// crossing bin holds more than `cap` elements or the table does not fit.
template <int DT, int NT>
__device__ bool finish_full(const GlobalSrc<DT, NT>& g, const tg_row_params& p, float u, BlockScratch& sm,
                            unsigned char* scratch, int cap, int& out_id, float& out_prob) {
  using E = Elt<DT>;
  constexpr int EPV = E::kEPV;
  const int t = threadIdx.x;
  const int niter = (g.nvec + NT - 1) / NT;
  if (niter > 4 * NT) return false;  // the table scan covers 4 iterations per thread
  float ymax = neg_inf();
  g.for_each([&](int, float y) { ymax = fmaxf(ymax, y); });
  ymax = block_max<NT>(ymax, sm);
  if (ymax == neg_inf()) { out_id = -1; out_prob = 0.0f; return true; }
  const float T = p.temperature;
  const float smax = __fdiv_rn(ymax, T);
  const float ylim = __fmul_rn(__fsub_rn(smax, 32.0f), T);  // zero mass at or below (see finish_row)
  const bool use_lim = fabsf(smax) < 1.0e5f;
  // mass and tempered value of value y (0 for -inf and provably zero masses)
  auto qs = [&](float y, float& sv) -> unsigned long long {
    if (!(y > neg_inf()) || (use_lim && !(y > ylim))) return 0ull;
    sv = __fdiv_rn(y, T);
    return qmass_le0(__fsub_rn(sv, smax));
  };
  auto dbin = [&](float sv) {
    const int bn = static_cast<int>(__fmul_rn(__fsub_rn(smax, sv), 32.0f));
    return bn > 1023 ? 1023 : bn;
  };
  float* my = reinterpret_cast<float*>(scratch);
  int* mid = reinterpret_cast<int*>(scratch + static_cast<size_t>(cap) * 4);

  const bool toppon = p.top_p < 1.0f;
  uint32_t cut_key = 0;
  int cut_id = 0x7fffffff;
  if (toppon) {
    hist_zero<NT, 1024, true>(sm);
    __syncthreads();
    unsigned long long Q = 0;
    g.for_each([&](int, float y) {
      float sv;
      const unsigned long long q = qs(y, sv);
      if (q) { Q += q; hist_put<true>(sm, dbin(sv), q); }
    });
    Q = block_sum<NT>(Q, sm);
    const double tau = __dmul_rn(static_cast<double>(p.top_p), __ull2double_rn(Q));
    if (!(tau > 0.0)) {  // the single top element: the smallest id holding the maximum
      cut_key = fkey(smax);
      unsigned int best = 0u;
      g.for_each([&](int v, float y) {
        if (y == ymax) best = max(best, ~static_cast<uint32_t>(v));
      });
      cut_id = static_cast<int>(~block_max_u32<NT>(best, sm));
    } else {
      const HistSel hs = hist_scan<NT, 1024, true>([&](unsigned long long m) { return __ull2double_rn(m) >= tau; }, sm);
      if (t == 0) sm.cand_count = 0;
      __syncthreads();
      g.for_each([&](int v, float y) {
        float sv;
        if (qs(y, sv) == 0 || dbin(sv) != hs.bin) return;
        const int pos = atomicAdd(&sm.cand_count, 1);
        if (pos < cap) { my[pos] = sv; mid[pos] = v; }
      });
      __syncthreads();
      const int m = sm.cand_count;
      __syncthreads();
      if (m > cap) return false;
      SmemSrcT<NT> ms{my, mid, m, neg_inf()};
      unsigned long long above = 0, qt = 0;
      unsigned int nties = 0, cb;
      unsigned long long jstar = 1;
      const unsigned long long before = hs.before;
      radix_find<NT, true, true>(
          ms, 32,
          [&](int, float sv, uint32_t& key, unsigned long long& w) {
            key = fkey(sv);
            w = qmass_le0(__fsub_rn(sv, smax));
            return true;
          },
          [&](unsigned long long mm, unsigned int) { return __ull2double_rn(before + mm) >= tau; }, sm,
          cut_key, above, cb, nties, qt);
      above += before;
      qt = qmass(__fsub_rn(key2f(cut_key), smax));
      if (qt > 0) {
        const double need = tau - __ull2double_rn(above);
        if (need > 0.0) {
          const double est = ceil(__ddiv_rn(need, __ull2double_rn(qt)));
          jstar = est < 1.0 ? 1ull : static_cast<unsigned long long>(est);
        }
        if (jstar > nties) jstar = nties;
        while (jstar > 1 && __ull2double_rn(above + (jstar - 1) * qt) >= tau) jstar--;
        while (jstar < nties && __ull2double_rn(above + jstar * qt) < tau) jstar++;
      }
      if (jstar < nties) {
        uint32_t idkey; unsigned long long b1, m1; unsigned int c1, n1;
        const unsigned int js = static_cast<unsigned int>(jstar);
        radix_find<NT, false, false>(
            ms, 20,
            [&](int id, float sv, uint32_t& key, unsigned long long& w) {
              if (fkey(sv) != cut_key) return false;
              key = static_cast<uint32_t>(id);
              w = 0;
              return true;
            },
            [&](unsigned long long, unsigned int c) { return c >= js; }, sm, idkey, b1, c1, n1, m1);
        cut_id = static_cast<int>(idkey);
      }
    }
  }
  const bool minpon = p.min_p > 0.0f;
  const double minq = __dmul_rn(static_cast<double>(fminf(p.min_p, 1.0f)), static_cast<double>(kMassScale));
  auto fin = [&](int v, float y) -> unsigned long long {  // final mass of element v
    float sv;
    const unsigned long long q = qs(y, sv);
    if (q == 0) return 0ull;
    if (toppon) {
      const uint32_t k = fkey(sv);
      if (k < cut_key || (k == cut_key && v > cut_id)) return 0ull;
    }
    return (!minpon || __ull2double_rn(q) >= minq) ? q : 0ull;
  };
  // pass 3: per-iteration sums (three 15/15/22-bit limbs of each warp's sum)
  unsigned int* tab = reinterpret_cast<unsigned int*>(scratch);
  __syncthreads();  // the member list is no longer needed
  for (int i = t; i < 3 * niter; i += NT) tab[i] = 0u;
  __syncthreads();
  unsigned long long sh = 0, sv8 = 0, stl = 0;
  if (t < g.head) sh = fin(t, g.value(t, E::load(g.row, t)));
  if (t < g.V - g.tail0) stl = fin(g.tail0 + t, g.value(g.tail0 + t, E::load(g.row, g.tail0 + t)));
  for (int it = 0; it < niter; it++) {
    const int j = it * NT + t;
    unsigned long long w = 0;
    if (j < g.nvec) {
      float y[EPV];
      g.vec(j, y);
#pragma unroll
      for (int e = 0; e < EPV; e++) w += fin(g.head + j * EPV + e, y[e]);
    }
    sv8 += w;
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(kFull, w, o);
    if ((t & 31) == 0 && w) {
      atomicAdd(&tab[it], static_cast<unsigned>(w & 0x7fffu));
      atomicAdd(&tab[niter + it], static_cast<unsigned>((w >> 15) & 0x7fffu));
      atomicAdd(&tab[2 * niter + it], static_cast<unsigned>(w >> 30));
    }
  }
  const unsigned long long H = block_sum<NT>(sh, sm);
  const unsigned long long S = block_sum<NT>(sh + sv8 + stl, sm);
  const unsigned long long r = draw_point(u, S);
  auto tab_at = [&](int it) {
    return static_cast<unsigned long long>(tab[it]) + (static_cast<unsigned long long>(tab[niter + it]) << 15) +
           (static_cast<unsigned long long>(tab[2 * niter + it]) << 30);
  };
  int pick = -1;
  unsigned long long qpick = 0;
  if (r < H) {  // in the scalar head: thread 0 scans it
    if (t == 0) {
      unsigned long long c = 0;
      for (int v = 0; v < g.head; v++) {
        const unsigned long long q = fin(v, g.value(v, E::load(g.row, v)));
        c += q;
        if (c > r) { pick = v; qpick = q; break; }
      }
      sm.sid[0] = pick; sm.sel_before = qpick;
    }
    __syncthreads();
    pick = sm.sid[0]; qpick = sm.sel_before;
    __syncthreads();
  } else {
    // the iteration holding r - H: a block scan over the table
    const unsigned long long r1 = r - H;
    constexpr int kPer = 4;
    unsigned long long loc = 0, vals[kPer];
#pragma unroll
    for (int k = 0; k < kPer; k++) {
      const int it = t * kPer + k;
      vals[k] = it < niter ? tab_at(it) : 0ull;
      loc += vals[k];
    }
    unsigned long long tot;
    const unsigned long long bef = block_excl_scan<NT>(loc, tot, sm);
    if (t == 0) { sm.sel_bin = 0xffffffffu; }
    __syncthreads();
    if (r1 >= bef && r1 < bef + loc) {
      unsigned long long c = bef;
#pragma unroll
      for (int k = 0; k < kPer; k++) {
        if (r1 < c + vals[k]) { sm.sel_bin = t * kPer + k; sm.sel_before = c; break; }
        c += vals[k];
      }
    }
    __syncthreads();
    const unsigned int its = sm.sel_bin;
    const unsigned long long ibefore = sm.sel_before;
    __syncthreads();
    if (its != 0xffffffffu) {
      const unsigned long long r2 = r1 - ibefore;
      const int j = static_cast<int>(its) * NT + t;
      float y[EPV];
      unsigned long long q8[EPV], w = 0;
      if (j < g.nvec) {
        g.vec(j, y);
#pragma unroll
        for (int e = 0; e < EPV; e++) { q8[e] = fin(g.head + j * EPV + e, y[e]); w += q8[e]; }
      }
      unsigned long long tw;
      const unsigned long long wb = block_excl_scan<NT>(w, tw, sm);
      if (w > 0 && r2 >= wb && r2 < wb + w) {
        unsigned long long c = wb;
#pragma unroll
        for (int e = 0; e < EPV; e++) {
          c += q8[e];
          if (c > r2) { sm.sid[0] = g.head + j * EPV + e; sm.sel_mass = q8[e]; break; }
        }
      }
      __syncthreads();
      pick = sm.sid[0];
      qpick = sm.sel_mass;
      __syncthreads();
    } else {  // past the vectors: the scalar tail, scanned by thread 0
      const unsigned long long r2 = r1 - tot;
      if (t == 0) {
        unsigned long long c = 0;
        for (int v = g.tail0; v < g.V; v++) {
          const unsigned long long q = fin(v, g.value(v, E::load(g.row, v)));
          c += q;
          if (c > r2) { pick = v; qpick = q; break; }
        }
        sm.sid[0] = pick; sm.sel_before = qpick;
      }
      __syncthreads();
      pick = sm.sid[0]; qpick = sm.sel_before;
      __syncthreads();
    }
  }
  out_id = pick;
  out_prob = __double2float_rn(__ddiv_rn(__ull2double_rn(qpick), __ull2double_rn(S)));
  return true;
}

// Survivors of the candidate path after compaction: slot i holds the tempered
// logit s (cand_y), the id (cand_id, -1 when dropped) and e = tg_exp(s - smax)
// (cand_e), so q = trunc(e * 2^44) needs no division or exponential.
template <int NT = kSampleNT>
struct ASrcT {
  const float* s;
  const int* id;
  int n;
  template <class F>
  __device__ __forceinline__ void for_each(F&& f) const {
    for (int i = threadIdx.x; i < n; i += NT)
      if (id[i] >= 0) f(i, s[i]);
  }
};

__device__ __forceinline__ unsigned long long mass_of_e(float e) {
  return __float2ull_rz(__fmul_rn(e, kMassScale));
}

// Stages (b)-(e) over the shared-memory candidate list (every element >= theta
// of the row).  Each selection is one wide histogram round over a monotone bin
// function; the crossing bin is then resolved exactly by one warp (<= 32
// members, the common case) or by the radix version above.  Returns false when
// an element below theta could survive top-k (the caller lowers theta).
// partial: the row has no top-k and the list holds only the elements >= theta;
// q_rest is then the exact mass of every other finite element.  The row can be
// finished from the list when the top-p cut falls inside it, or when min-p
// provably drops everything below theta; otherwise false.
template <int NT = kSampleNT>
__device__ bool finish_cands(float* cy, int* cid, float* ce, int n, float theta,
                             const tg_row_params& p, int V, float u, BlockScratch& sm,
                             int& out_id, float& out_prob, PhaseClock& pc, bool partial = false,
                             unsigned long long q_rest = 0, float below_override = 0.0f,
                             bool use_below = false, bool have_range = false, float ymax_in = 0.0f,
                             float nymin_in = 0.0f) {
  SmemSrcT<NT> src{cy, cid, n, theta};
  if (!(p.temperature > 0.0f)) return finish_row<NT>(src, p, V, u, false, theta, sm, out_id, out_prob);
  const float T = p.temperature;
  const bool topk = p.top_k > 0 && p.top_k < V;
  const int lane = threadIdx.x & 31;

  // largest value and minus the smallest finite one over the list (given by
  // the caller when it already reduced them)
  float ymax = ymax_in, nymin = nymin_in;
  if (!have_range) {
    ymax = neg_inf();
    nymin = neg_inf();
    src.for_each([&](int, float y) {
      ymax = fmaxf(ymax, y);
      if (y > neg_inf()) nymin = fmaxf(nymin, -y);
    });
    block_max2<NT>(ymax, nymin, sm);
  }
  const float ymin = -nymin;
  if (ymax == neg_inf()) { out_id = -1; out_prob = 0.0f; return !partial; }
  // an upper bound of the values absent from the list
  const float below = use_below ? below_override : key2f(fkey(theta) - 1u);
  // elements below theta must come strictly after the list in (s desc) order
  if (partial && __fdiv_rn(below, T) >= __fdiv_rn(ymin, T)) return false;

  float sk = neg_inf();
  if (topk) {
    const unsigned int k = static_cast<unsigned int>(p.top_k);
    const float width = __fsub_rn(ymax, ymin);
    const float scale = width > 0.0f ? __fdiv_rn(2046.0f, width) : 0.0f;
    auto binf = [&](float y) {  // descending y -> ascending bin; -inf last
      if (!(y > neg_inf())) return 2047;
      const int bn = static_cast<int>(__fmul_rn(__fsub_rn(ymax, y), scale));
      return bn > 2046 ? 2046 : bn;
    };
    const HistSel hs = hist_round<NT, 2048, false>(
        src, [&](int, float y, int& bin, unsigned long long& w) { bin = binf(y); w = 1; return true; },
        [&](unsigned long long c) { return c >= k; }, sm);
    if (hs.bin < 0) return false;
    const unsigned int j = k - static_cast<unsigned int>(hs.before);  // rank inside the bin
    const int nb = collect_small<NT>(
        src,
        [&](int i, float y, unsigned long long& key, unsigned long long& w, int& id) {
          if (binf(y) != hs.bin) return false;
          key = (static_cast<unsigned long long>(~fkey(y)) << 32) | static_cast<uint32_t>(i);
          w = 1;
          id = i;
          return true;
        },
        sm);
    uint32_t kkey;
    if (nb <= 32) {
      if (threadIdx.x < 32) {
        unsigned long long key, w;
        int id;
        warp_sorted_pick(nb, 0ull, [&](unsigned long long c) { return c >= j; }, sm, key, w, id);
        if (lane == 0) sm.sel_cnt = ~static_cast<uint32_t>(key >> 32);
      }
      __syncthreads();
      kkey = sm.sel_cnt;
      __syncthreads();
    } else {
      unsigned int lo = 0u, hi = 0u;  // max of ~key and of key over the bin
      src.for_each([&](int, float y) {
        if (binf(y) == hs.bin) { lo = max(lo, ~fkey(y)); hi = max(hi, fkey(y)); }
      });
      lo = ~block_max_u32<NT>(lo, sm);
      hi = block_max_u32<NT>(hi, sm);
      if (lo == hi) {
        kkey = hi;
      } else {
        unsigned long long b0, m0; unsigned int c0, n0;
        auto kw = [&](int, float y, uint32_t& key, unsigned long long& w) {
          if (binf(y) != hs.bin) return false;
          key = fkey(y); w = 0; return true;
        };
        auto rc = [&](unsigned long long, unsigned int c) { return c >= j; };
        radix_find<NT, true, false, SmemSrcT<NT>, decltype(kw), decltype(rc), true>(
            src, 32, kw, rc, sm, kkey, b0, c0, n0, m0);
      }
    }
    sk = __fdiv_rn(key2f(kkey), T);
    if ((use_below || theta > neg_inf()) && __fdiv_rn(below, T) >= sk) return false;
  }
  pc.mark(5);
  const float smax = __fdiv_rn(ymax, T);
  const bool minpon = p.min_p > 0.0f;
  const double minq = __dmul_rn(static_cast<double>(fminf(p.min_p, 1.0f)),
                                static_cast<double>(kMassScale));
  // partial rows: whether min-p drops every element below theta (tg_exp is
  // within one ulp of exp, hence the small relative margin)
  const bool minp_excludes_rest =
      minpon && __dadd_rn(__dmul_rn(__ull2double_rn(qmass(__fsub_rn(__fdiv_rn(below, T), smax))), 1.000001), 1.0) < minq;
  if (partial && p.top_p >= 1.0f && !minp_excludes_rest) return false;

  // compaction: s, e in place; ids of dropped slots set to -1.  The same pass
  // fills the top-p mass histogram over d = smax - s (32 bins per unit of s).
  const bool toppon = p.top_p < 1.0f;
  auto dbin = [&](float sv) {
    const int bn = static_cast<int>(__fmul_rn(__fsub_rn(smax, sv), 32.0f));
    return bn > 1023 ? 1023 : bn;
  };
  if (toppon) hist_zero<NT, 1024, true>(sm);
  __syncthreads();
  unsigned long long Q = 0;
  for (int i = threadIdx.x; i < n; i += NT) {
    const float y = cy[i];
    bool keep = cid[i] >= 0 && y >= theta && y > neg_inf();
    float sv = 0.0f, e = 0.0f;
    if (keep) {
      sv = __fdiv_rn(y, T);
      keep = !topk || sv >= sk;
    }
    if (keep) {
      const float d = __fsub_rn(sv, smax);
      e = d >= -32.0f ? tg_exp(d) : 0.0f;
      const unsigned long long q = mass_of_e(e);
      Q += q;
      if (toppon && q > 0) hist_put<true>(sm, dbin(sv), q);
      cy[i] = sv;
      ce[i] = e;
    } else {
      cid[i] = -1;
    }
  }
  Q = block_sum<NT>(Q, sm) + q_rest;
  ASrcT<NT> as{cy, cid, n};
  pc.mark(6);

  // (d) top-p: the last element (cut_key, cut_id) of the shortest prefix in
  // (s desc, id asc) order whose mass reaches top_p * Q.
  uint32_t cut_key = 0;
  int cut_id = 0x7fffffff;
  if (toppon) {
    const double tau = __dmul_rn(static_cast<double>(p.top_p), __ull2double_rn(Q));
    bool resolved = false;
    if (tau > 0.0) {
      const HistSel hs = hist_scan<NT, 1024, true>(
          [&](unsigned long long m) { return __ull2double_rn(m) >= tau; }, sm);
      if (hs.bin >= 0) {
        const int nb = collect_small<NT>(
            as,
            [&](int i, float sv, unsigned long long& key, unsigned long long& w, int& id) {
              w = mass_of_e(ce[i]);
              if (w == 0 || dbin(sv) != hs.bin) return false;
              id = cid[i];
              key = (static_cast<unsigned long long>(~fkey(sv)) << 32) | static_cast<uint32_t>(id);
              return true;
            },
            sm);
        if (nb <= 32) {
          if (threadIdx.x < 32) {
            unsigned long long key, w;
            int id;
            warp_sorted_pick(nb, hs.before, [&](unsigned long long m) { return __ull2double_rn(m) >= tau; },
                             sm, key, w, id);
            if (lane == 0) { sm.sel_cnt = ~static_cast<uint32_t>(key >> 32); sm.sid[0] = id; }
          }
          __syncthreads();
          cut_key = sm.sel_cnt;
          cut_id = sm.sid[0];
          __syncthreads();
          resolved = true;
        }
      } else if (partial) {  // the prefix runs past the list
        if (!minp_excludes_rest) return false;
        cut_key = 0u;  // every list element is inside the prefix
        cut_id = 0x7fffffff;
        resolved = true;
      }
    } else {  // top_p <= 0: the single top element (smallest id among the maxima)
      cut_key = fkey(smax);
      unsigned int best = 0u;
      as.for_each([&](int i, float sv) {
        if (fkey(sv) == cut_key) best = max(best, ~static_cast<uint32_t>(cid[i]));
      });
      cut_id = static_cast<int>(~block_max_u32<NT>(best, sm));
      resolved = true;
    }
    if (!resolved) {  // crowded bin: exact radix over the whole survivor set
      unsigned long long above = 0, qt = 0;
      unsigned int nties = 0, cb;
      unsigned long long jstar = 1;
      radix_find<NT, true, true>(
          as, 32,
          [&](int i, float sv, uint32_t& key, unsigned long long& w) {
            key = fkey(sv);
            w = mass_of_e(ce[i]);
            return true;
          },
          [&](unsigned long long m, unsigned int) { return __ull2double_rn(m) >= tau; }, sm,
          cut_key, above, cb, nties, qt);
      qt = qmass(__fsub_rn(key2f(cut_key), smax));
      if (qt > 0) {
        const double need = tau - __ull2double_rn(above);
        if (need > 0.0) {
          const double est = ceil(__ddiv_rn(need, __ull2double_rn(qt)));
          jstar = est < 1.0 ? 1ull : static_cast<unsigned long long>(est);
        }
        if (jstar > nties) jstar = nties;
        while (jstar > 1 && __ull2double_rn(above + (jstar - 1) * qt) >= tau) jstar--;
        while (jstar < nties && __ull2double_rn(above + jstar * qt) < tau) jstar++;
      }
      if (jstar < nties) {
        uint32_t idkey; unsigned long long b1, m1; unsigned int c1, n1;
        const unsigned int js = static_cast<unsigned int>(jstar);
        radix_find<NT, false, false>(
            as, 20,
            [&](int i, float sv, uint32_t& key, unsigned long long& w) {
              if (fkey(sv) != cut_key) return false;
              key = static_cast<uint32_t>(cid[i]);
              w = 0;
              return true;
            },
            [&](unsigned long long, unsigned int c) { return c >= js; }, sm, idkey, b1, c1, n1, m1);
        cut_id = static_cast<int>(idkey);
      }
    }
  }
  pc.mark(7);
  const int idbits = 32 - __clz(V > 1 ? V - 1 : 1);
  const int shift = idbits > 10 ? idbits - 10 : 0;
  hist_zero<NT, 1024, true>(sm);
  __syncthreads();
  unsigned long long S = 0;  // the same pass fills the draw histogram over id bins
  for (int i = threadIdx.x; i < n; i += NT) {
    const int id = cid[i];
    if (id < 0) continue;
    const unsigned long long q = mass_of_e(ce[i]);
    bool keep = true;
    if (toppon) {
      const uint32_t k = fkey(cy[i]);
      keep = k > cut_key || (k == cut_key && id <= cut_id);
    }
    if (keep && minpon) keep = __ull2double_rn(q) >= minq;
    if (keep) {
      S += q;
      if (q > 0) hist_put<true>(sm, id >> shift, q);
    } else {
      cid[i] = -1;
    }
  }
  S = block_sum<NT>(S, sm);
  pc.mark(8);

  // (e) draw: first id in index order whose running mass exceeds r
  const unsigned long long r = draw_point(u, S);
  const HistSel hd = hist_scan<NT, 1024, true>([&](unsigned long long m) { return m > r; }, sm);
  int pick = -1;
  unsigned long long qpick = 0;
  if (hd.bin >= 0) {
    const int nb = collect_small<NT>(
        as,
        [&](int i, float, unsigned long long& key, unsigned long long& w, int& id) {
          w = mass_of_e(ce[i]);
          id = cid[i];
          if (w == 0 || (id >> shift) != hd.bin) return false;
          key = static_cast<unsigned long long>(id);
          return true;
        },
        sm);
    if (nb <= 32) {
      if (threadIdx.x < 32) {
        unsigned long long key, w;
        int id;
        warp_sorted_pick(nb, hd.before, [&](unsigned long long m) { return m > r; }, sm, key, w, id);
        if (lane == 0) { sm.sid[0] = id; sm.sel_before = w; }
      }
      __syncthreads();
      pick = sm.sid[0];
      qpick = sm.sel_before;
      __syncthreads();
    }
  }
  if (pick < 0) {
    uint32_t pk; unsigned long long b2, qp; unsigned int c2, n2;
    radix_find<NT, false, true>(
        as, 20,
        [&](int i, float, uint32_t& key, unsigned long long& w) {
          key = static_cast<uint32_t>(cid[i]);
          w = mass_of_e(ce[i]);
          return true;
        },
        [&](unsigned long long m, unsigned int) { return m > r; }, sm, pk, b2, c2, n2, qp);
    pick = static_cast<int>(pk);
    qpick = qp;
  }
  pc.mark(9);
  out_id = pick;
  out_prob = __double2float_rn(__ddiv_rn(__ull2double_rn(qpick), __ull2double_rn(S)));
  return true;
}

// Threshold from the per-vector maxima of the sample: one histogram round over
// bins of equal width between the largest and the smallest finite maximum,
// then the smallest maximum inside the bin that holds the rk-th largest (a
// lower bound of the rk-th largest; -inf when rk exceeds the sample).
template <int N, int NT = kSampleNT, int BAR = 0>
__device__ float sample_theta(const float* vm, unsigned int rk, BlockScratch& sm) {
  float mx = neg_inf(), nmn = neg_inf();
#pragma unroll
  for (int i = 0; i < N; i++) {
    mx = fmaxf(mx, vm[i]);
    if (vm[i] > neg_inf()) nmn = fmaxf(nmn, -vm[i]);
  }
  block_max2<NT, BlockScratch, BAR>(mx, nmn, sm);
  const float mn = -nmn;
  if (mx == neg_inf()) return neg_inf();
  const float width = __fsub_rn(mx, mn);
  const float scale = width > 0.0f ? __fdiv_rn(2046.0f, width) : 0.0f;
  auto binf = [&](float v) {
    if (!(v > neg_inf())) return 2047;
    const int bn = static_cast<int>(__fmul_rn(__fsub_rn(mx, v), scale));
    return bn > 2046 ? 2046 : bn;
  };
  auto bw = [&](int, float v, int& bin, unsigned long long& w) { bin = binf(v); w = 1; return true; };
  auto reached = [&](unsigned long long c) { return c >= rk; };
  const HistSel hs = hist_round<NT, 2048, false, RegSrc<N>, decltype(bw), decltype(reached), BAR>(RegSrc<N>{vm}, bw, reached, sm);
  if (hs.bin < 0 || hs.bin == 2047) return neg_inf();
  float nlo = neg_inf();
#pragma unroll
  for (int i = 0; i < N; i++)
    if (binf(vm[i]) == hs.bin) nlo = fmaxf(nlo, -vm[i]);
  return -block_max<NT, BlockScratch, BAR>(nlo, sm);
}

// Vocab-sharded mode, local half: the record of one row -- every local value
// >= the local k-th value (ties kept; for greedy rows the local first maximum)
// with global ids.  Rows that are neither greedy nor top-k <= kFastMaxK get
// count -1.
// `below`: an upper bound of the local values the source does not yield.
template <int NT = kSampleNT, class Src>
__device__ void shard_emit(const Src& src, const tg_row_params& p, int V, int moff,
                           tg_shard_record* rec, BlockScratch& sm, float below) {
  const int t = threadIdx.x;
  const bool greedy = !(p.temperature > 0.0f);
  if (greedy) {
    float y = neg_inf();
    int id = 0x7fffffff;
    src.for_each([&](int i, float v) {
      if (v > y || (v == y && i < id)) { y = v; id = i; }
    });
    block_argmax<NT>(y, id, sm);
    if (t == 0) {
      rec->flags = 0;
      rec->absent_max = neg_inf();
      rec->count = id == 0x7fffffff ? 0 : 1;
      if (id != 0x7fffffff) { rec->cand[0].value = y; rec->cand[0].id = id + moff; }
    }
    return;
  }
  if (!(p.top_k > 0 && p.top_k <= kFastMaxK)) {
    if (t == 0) { rec->count = -1; rec->flags = 0; }
    return;
  }
  float kth = neg_inf();
  if (p.top_k < V) {
    uint32_t kkey; unsigned long long b0, m0; unsigned int c0, n0;
    const unsigned int k = static_cast<unsigned int>(p.top_k);
    auto kw = [&](int, float y, uint32_t& key, unsigned long long& w) { key = fkey(y); w = 0; return true; };
    auto rc = [&](unsigned long long, unsigned int c) { return c >= k; };
    radix_find<NT, true, false, Src, decltype(kw), decltype(rc), true>(src, 32, kw, rc, sm, kkey, b0, c0, n0, m0);
    kth = key2f(kkey);
  }
  if (t == 0) sm.sn = 0;
  __syncthreads();
  float absent = below;
  src.for_each([&](int i, float y) {
    if (y >= kth && y > neg_inf()) {
      const int pos = atomicAdd(&sm.sn, 1);
      if (pos < TG_SHARD_CAP) { rec->cand[pos].value = y; rec->cand[pos].id = i + moff; }
    } else {
      absent = fmaxf(absent, y);
    }
  });
  absent = block_max<NT>(absent, sm);
  if (t == 0) {
    const int c = sm.sn;
    rec->count = c < TG_SHARD_CAP ? c : TG_SHARD_CAP;
    rec->flags = c > TG_SHARD_CAP ? 1 : 0;
    rec->absent_max = absent;
  }
  __syncthreads();
}

// kStream: the streaming half of the two-kernel mode (threshold, streaming
// pass, raw candidates to global memory); no history, no selection code.
template <int DT, bool kStream, int NT>
__device__ __forceinline__ void sample_row(const SampleArgs& a, const int b) {
  using E = Elt<DT>;
  constexpr int EPV = E::kEPV;
  constexpr int SV = kSampleVecs;
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ BlockScratch sm;
  __shared__ uint32_t bloom[128];
  const int t = threadIdx.x;
  const int moff = a.vocab_offset;  // global id of this shard's element 0
  const int V = a.vocab;
  float* cand_y;
  int* cand_id;
  float* cand_e;
  if constexpr (kStream) {  // list in global memory; the warps' rings are the shared memory
    cand_y = a.cand_gy + static_cast<int64_t>(b) * kCandMax;
    cand_id = a.cand_gid + static_cast<int64_t>(b) * kCandMax;
    cand_e = reinterpret_cast<float*>(dyn);
  } else {
    cand_y = reinterpret_cast<float*>(dyn);
    cand_id = reinterpret_cast<int*>(dyn + kCandMax * 4);
    cand_e = reinterpret_cast<float*>(dyn + kCandMax * 8);
  }
  int* hkey = reinterpret_cast<int*>(dyn + kCandMax * 12);
  const int ht = a.ht_log2 ? (1 << a.ht_log2) : 0;
  int* hval = hkey + ht;

  PhaseClock pc;
  pc.row = b;
  pc.mark(0);
  const tg_row_params p = a.params[b];
  const char* row = reinterpret_cast<const char*>(a.logits) + b * a.row_stride * E::kSize;
  const float u = a.uniforms ? a.uniforms[b] : 0.0f;

  const uint32_t* mask = nullptr;
  if (a.mask_table && a.state_id) {
    const int sid = a.state_id[b];
    if (sid >= a.num_states) {
      if constexpr (kStream) {  // the finishing kernel reports it
        if (t == 0) a.cand_gn[b] = -1;
        return;
      }
      if (t == 0) {
        if (a.shard_out) {
          a.shard_out[b].count = -1;
          a.shard_out[b].flags = 0;
        } else {
          a.out_ids[b] = -1;
          if (a.out_probs) a.out_probs[b] = 0.0f;
        }
        atomicOr(a.status, 1u);
      }
      return;
    }
    if (sid >= 0) mask = a.mask_table + static_cast<int64_t>(sid) * a.mask_words;
  }

  // row geometry: scalar head up to the first 16-byte boundary, vectors, tail
  const uintptr_t addr = reinterpret_cast<uintptr_t>(row);
  int head = static_cast<int>(((16u - (addr & 15u)) & 15u) / E::kSize);
  if (head > V) head = V;
  const int nvec = (V - head) / EPV;
  const int tail0 = head + nvec * EPV;
  const uint4* vrow = reinterpret_cast<const uint4*>(row + head * E::kSize);

  int hlen = 0;
  if (a.history_len && a.history && a.hist_cap > 0) {
    hlen = a.history_len[b];
    hlen = hlen < 0 ? 0 : (hlen > a.hist_cap ? a.hist_cap : hlen);
  }
  const bool rep_on = p.repetition_penalty > 1.0f;
  const bool pf_on = p.presence_penalty != 0.0f || p.frequency_penalty != 0.0f;
  Hist hist{hkey, hval, bloom, ht - 1, a.ht_log2, 0};
  const bool need_hist = !kStream && hlen > 0 && (rep_on || pf_on);

  // (a) history -> shared hash of penalised values (raw values read from L2
  // when this runs after the streaming pass)
  // Penalty of one history token (raw value already masked), count c.
  auto penalise = [&](float y, int c) {
    if (y == neg_inf()) return y;
    if (rep_on) y = y > 0.0f ? __fdiv_rn(y, p.repetition_penalty) : __fmul_rn(y, p.repetition_penalty);
    if (pf_on) y = __fsub_rn(y, __fadd_rn(__fmul_rn(p.frequency_penalty, static_cast<float>(c)), p.presence_penalty));
    return y;
  };
  // Penalties can raise a logit only through a negative presence / frequency.
  const bool risers = pf_on && (p.presence_penalty < 0.0f || p.frequency_penalty < 0.0f);
  bool hist_counts_only = false;

  // build_hist(th, values): hash of the distinct history ids with their counts.
  // With values, every slot also gets its penalised value (raw value read from
  // global memory) and ids whose penalised value reaches th while the raw one
  // did not are appended to the candidate list; without, slots keep counts and
  // the candidate list is penalised from its own raw values.
  auto build_hist = [&](float th, bool values) {
    if (!need_hist || hist.active) return;
    for (int i = t; i < ht; i += NT) { hkey[i] = -1; hval[i] = 0; }
    for (int i = t; i < 128; i += NT) bloom[i] = 0u;
    __syncthreads();
    const int32_t* h = a.history + static_cast<int64_t>(b) * a.history_stride;
    for (int i = t; i < hlen; i += NT) {
      const int id = h[i] - moff;  // history ids are global
      if (id < 0 || id >= V) continue;
      int s = hist.slot0(id);
      for (;;) {
        const int old = atomicCAS(&hkey[s], -1, id);
        if (old == -1 || old == id) { atomicAdd(&hval[s], 1); break; }
        s = (s + 1) & (ht - 1);
      }
    }
    __syncthreads();
    for (int s = t; s < ht; s += NT) {
      const int id = hkey[s];
      if (id < 0) continue;
      const uint32_t hb = Hist::bloom_bit(id);
      atomicOr(&bloom[hb >> 5], 1u << (hb & 31));
      if (!values) continue;
      float raw = E::load(row, id);
      if (mask && !mask_allows(mask, moff + id)) raw = neg_inf();
      const float y = penalise(raw, hval[s]);
      hval[s] = __float_as_int(y);
      if (!(raw >= th) && y >= th) {
        const int pos = atomicAdd(&sm.cand_count, 1);
        if (pos < kCandMax) { cand_y[pos] = y; cand_id[pos] = id; }
      }
    }
    hist.active = 1;
    hist_counts_only = !values;
    __syncthreads();
  };

  const bool greedy = !(p.temperature > 0.0f);
  const bool topk = p.top_k > 0 && p.top_k < V;
  // rows without top-k but with top-p / min-p: the list holds the largest
  // ~kNoTopkTarget values and the rest of the row contributes its mass only
  const bool truncated = p.top_p < 1.0f || p.min_p > 0.0f;
  const bool fast = greedy || (topk && p.top_k <= kFastMaxK) || V <= kCandMax || (!topk && truncated);
  int out_id = -1;
  float out_prob = 0.0f;
  bool done = false;
  if constexpr (kStream) {
    if (!fast) {
      if (t == 0) a.cand_gn[b] = -1;
      return;
    }
  }
  // two-kernel mode: this row's candidates were streamed already
  const bool pre = !kStream && a.cand_gn != nullptr && a.cand_gn[b] >= 0;

  if (fast) {
    const int keff = greedy ? 1 : (topk ? p.top_k : V);
    const unsigned int need = static_cast<unsigned int>(keff < V ? keff : 1);
    const float tgt =
        kTgtMul * static_cast<float>(keff < V ? keff : (kStream || NT == kSampleNT ? kNoTopkTargetStream : kNoTopkTarget)) +
        kTgtAdd;
    const int lane = t & 31, warp = t >> 5;
    const unsigned lt = (1u << lane) - 1u;

    auto vmax_of = [&](const uint4& w, int j) {
      if (!mask) return E::vmax(w);
      float x[EPV];
      E::unpack(w, x);
      const uint32_t bits = mask_bits(mask, moff + head + j * EPV, EPV);
      float vm = neg_inf();
#pragma unroll
      for (int e = 0; e < EPV; e++)
        if ((bits >> e) & 1u) vm = fmaxf(vm, x[e]);
      return vm;
    };
    // Append the elements >= th of vector j (raw w) to the candidate list.
    auto append_vec = [&](const uint4& w, int j, float th) {
      float x[EPV];
      E::unpack(w, x);
      const uint32_t bits = mask ? mask_bits(mask, moff + head + j * EPV, EPV) : 0xffu;
      uint32_t hits = 0;
#pragma unroll
      for (int e = 0; e < EPV; e++) hits |= (((bits >> e) & 1u) && x[e] >= th ? 1u : 0u) << e;
      if (!hits) return;
      int pos = atomicAdd(&sm.cand_count, __popc(hits));
#pragma unroll
      for (int e = 0; e < EPV; e++) {
        if ((hits >> e) & 1u) {
          if (pos < kCandMax) { cand_y[pos] = x[e]; cand_id[pos] = head + j * EPV + e; }
          pos++;
        }
      }
    };
    auto scalars = [&](float th) {
      int sc_id = -1;
      if (t < head) sc_id = t;
      else if (t - head < V - tail0) sc_id = tail0 + (t - head);
      if (sc_id < 0) return;
      float sc = E::load(row, sc_id);
      if (mask && !mask_allows(mask, moff + sc_id)) sc = neg_inf();
      if (sc >= th) {
        const int pos = atomicAdd(&sm.cand_count, 1);
        if (pos < kCandMax) { cand_y[pos] = sc; cand_id[pos] = sc_id; }
      }
    };
    // Per-warp ring of hit vectors (raw 16 bytes + vector index) in the bytes
    // of cand_e, which stage (b) only needs later.  A warp drains its ring
    // itself whenever it holds >= 32 entries: lane i expands entries i, i+32.
    // (wide CTAs: the rings get their own shared memory after the hash)
    uint4* rbase = reinterpret_cast<uint4*>(cand_e);
    if constexpr (!kStream && (NT / 32) * kRing * 20 > kCandMax * 4)
      rbase = reinterpret_cast<uint4*>(dyn + kCandMax * 12 + (ht ? static_cast<size_t>(8) * ht : 0));
    constexpr int RING = kStream ? kStreamRing : kRing;
    uint4* rdata = rbase + warp * RING;
    int* ridx = reinterpret_cast<int*>(rbase + (NT / 32) * RING) + warp * RING;
    auto drain = [&](int cnt, float th) {  // warp-uniform cnt <= RING
      __syncwarp();
      for (int i0 = 0; i0 < cnt; i0 += 32) {
        const int i = i0 + lane;
        float x[EPV];
        uint32_t hits = 0;
        int j = 0;
        if (i < cnt) {
          j = ridx[i];
          E::unpack(rdata[i], x);
          const uint32_t bits = mask ? mask_bits(mask, moff + head + j * EPV, EPV) : 0xffu;
#pragma unroll
          for (int e = 0; e < EPV; e++) hits |= (((bits >> e) & 1u) && x[e] >= th ? 1u : 0u) << e;
        }
        const int c = __popc(hits);
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += v;
        }
        const int tot = __shfl_sync(kFull, incl, 31);
        int base = 0;
        if (lane == 31 && tot) base = atomicAdd(&sm.cand_count, tot);
        int pos = __shfl_sync(kFull, base, 31) + incl - c;
        // a lane's hits, one set bit at a time (usually one or two of EPV)
        while (hits) {
          const int e = __ffs(hits) - 1;
          hits &= hits - 1u;
          float xe = x[0];
#pragma unroll
          for (int f = 1; f < EPV; f++) xe = e == f ? x[f] : xe;  // register select, no local memory
          if (pos < kCandMax) { cand_y[pos] = xe; cand_id[pos] = head + j * EPV + e; }
          pos++;
        }
      }
      __syncwarp();
    };
    // The streaming pass: one 128-bit load, a vector max and a compare per 16
    // bytes; a warp ballot sends the vectors holding an element >= th to the ring.
    auto scan = [&](float th, int j0) {
      int rcnt = 0;  // warp-uniform ring fill
      // exact per-vector test of one group; hit vectors go to the ring
      auto group = [&](const uint4* w, int jb) {
#pragma unroll
        for (int q = 0; q < kUnroll; q++) {
          if (jb + q * NT >= nvec) break;  // warp-uniform
          const int j = jb + q * NT + t;
          const bool hit = j < nvec && vmax_of(w[q], j) >= th;
          const unsigned bal = __ballot_sync(kFull, hit);
          if (bal) {
            if (hit) {
              const int pos = rcnt + __popc(bal & lt);
              rdata[pos] = w[q];
              ridx[pos] = j;
            }
            rcnt += __popc(bal);
            if (rcnt >= 32) { drain(rcnt, th); rcnt = 0; }
          }
        }
      };
      int jb = j0;
      if (!mask && kStream) {
        // full groups of the streaming kernel: each vector's maximum once, a
        // 4-bit hit mask per thread and one warp prefix sum place the hit
        // vectors in the ring (a warp group holds a hit ~85 % of the time on
        // config 4, so a per-warp skip test rarely pays)
        for (; jb + kUnroll * NT <= nvec; jb += kUnroll * NT) {
          const uint4* pv = vrow + jb + t;
          uint4 w[kUnroll];
#pragma unroll
          for (int q = 0; q < kUnroll; q++) w[q] = ldg_stream(pv + q * NT);
          unsigned hm = 0;
#pragma unroll
          for (int q = 0; q < kUnroll; q++) hm |= (E::vmax(w[q]) >= th ? 1u : 0u) << q;
          const int c = __popc(hm);
          int incl = c;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += v;
          }
          const int total = __shfl_sync(kFull, incl, 31);
          if (total) {
            int pos = rcnt + incl - c;
#pragma unroll
            for (int q = 0; q < kUnroll; q++) {
              if ((hm >> q) & 1u) {
                rdata[pos] = w[q];
                ridx[pos] = jb + q * NT + t;
                pos++;
              }
            }
            rcnt += total;
            if (rcnt >= 32) { drain(rcnt, th); rcnt = 0; }
          }
        }
      } else if (!mask) {
        // full groups: no bounds checks, and one packed max over the lane's
        // vectors decides whether the warp needs the exact per-vector test
        for (; jb + kUnroll * NT <= nvec; jb += kUnroll * NT) {
          const uint4* pv = vrow + jb + t;
          uint4 w[kUnroll];
#pragma unroll
          for (int q = 0; q < kUnroll; q++) w[q] = ldg_stream(pv + q * NT);
          if (__any_sync(kFull, E::template vmax_n<kUnroll>(w) >= th)) group(w, jb);
        }
      }
      for (; jb < nvec; jb += kUnroll * NT) {
        uint4 w[kUnroll];
#pragma unroll
        for (int q = 0; q < kUnroll; q++) {
          const int j = jb + q * NT + t;
          if (j < nvec) w[q] = ldg_stream(vrow + j);
        }
        group(w, jb);
      }
      if (rcnt) drain(rcnt, th);
    };
    auto expand = [&](float) {
      __syncthreads();
      return true;
    };

    // Sample: the first SV vectors of every thread; their per-vector maxima
    // give the threshold for the rest of the row.
    const int nsv = nvec < SV * NT ? nvec : SV * NT;
    const int sampled = nsv * EPV;
    auto rank_for = [&](float mult) {
      int rr = static_cast<int>(ceilf(mult * tgt * static_cast<float>(sampled > 0 ? sampled : 1) /
                                      static_cast<float>(V)));
      return static_cast<unsigned int>(rr < 1 ? 1 : rr);
    };
    float theta = neg_inf();
    unsigned int rk = 0;
    bool fits;
    bool fused = false;  // list penalised, counted and its range reduced on load
    unsigned int f_cnt = 0;
    float f_ymax = neg_inf(), f_nymin = neg_inf();
    if (pre) {
      pc.mark(0);
      if (V > kCandMax && sampled > 0) rk = rank_for(1.0f);
      theta = a.cand_gth[b];
      const int n = a.cand_gn[b];
      const int m = n < kCandMax ? n : kCandMax;
      const float* gy = a.cand_gy + static_cast<int64_t>(b) * kCandMax;
      const int* gid = a.cand_gid + static_cast<int64_t>(b) * kCandMax;
      // the list arrives with the penalties applied, counted and with its range
      // reduced in one pass (when penalties cannot raise a value); the first
      // batch of loads is issued before the history hash is built
      fused = !(need_hist && risers);
      constexpr int LU = 4;
      float yv[LU];
      int iv[LU];
      auto load_batch = [&](int base) {
#pragma unroll
        for (int q = 0; q < LU; q++) {
          const int i = base + q * NT + t;
          if (i < m) { yv[q] = __ldcs(gy + i); iv[q] = __ldcs(gid + i); }
        }
      };
      load_batch(0);
      if (!risers) build_hist(0.0f, false);
      unsigned long long cnt = 0;
      float ymx = neg_inf(), nymn = neg_inf();
      for (int base = 0; base < m; base += LU * NT) {
        if (base > 0) load_batch(base);
#pragma unroll
        for (int q = 0; q < LU; q++) {
          const int i = base + q * NT + t;
          if (i >= m) break;
          float y = yv[q];
          const int id = iv[q];
          float hv;
          if (fused && hist_counts_only && hist.find(id, hv)) y = penalise(y, __float_as_int(hv));
          cand_y[i] = y;
          cand_id[i] = id;
          if (id >= 0 && y >= theta) {
            cnt++;
            ymx = fmaxf(ymx, y);
            if (y > neg_inf()) nymn = fmaxf(nymn, -y);
          }
        }
      }
      if (t == 0) sm.cand_count = n;
      if (fused) {  // one reduction of the three (its barriers also publish the list)
        for (int o = 16; o > 0; o >>= 1) {
          cnt += __shfl_xor_sync(kFull, cnt, o);
          ymx = fmaxf(ymx, __shfl_xor_sync(kFull, ymx, o));
          nymn = fmaxf(nymn, __shfl_xor_sync(kFull, nymn, o));
        }
        if ((t & 31) == 0) { sm.red_u64[t >> 5] = cnt; sm.red_f[t >> 5] = ymx; sm.red_f2[t >> 5] = nymn; }
        __syncthreads();
        f_cnt = 0;
        f_ymax = neg_inf();
        f_nymin = neg_inf();
#pragma unroll
        for (int i = 0; i < NT / 32; i++) {
          f_cnt += static_cast<unsigned int>(sm.red_u64[i]);
          f_ymax = fmaxf(f_ymax, sm.red_f[i]);
          f_nymin = fmaxf(f_nymin, sm.red_f2[i]);
        }
      }
      __syncthreads();
      fits = true;
      pc.mark(1);
    } else if (kStream && a.theta_given) {
      // theta from theta_kernel: the stream starts on its loads at once
      if (V > kCandMax && sampled > 0) rk = rank_for(1.0f);
      theta = a.cand_gth[b];
      if (t == 0) sm.cand_count = 0;
      __syncthreads();
      pc.mark(1);
      scalars(theta);
      scan(theta, 0);
      fits = expand(theta);
    } else {
      uint4 raw[SV];
      float vm[SV];
      pc.mark(0);
#pragma unroll
      for (int q = 0; q < SV; q++) {
        const int j = t + q * NT;
        if (j < nvec) raw[q] = ldg_stream(vrow + j);
      }
      // the history hash (counts only) is built while the sample loads fly
      if (!risers) build_hist(0.0f, false);
#pragma unroll
      for (int q = 0; q < SV; q++) {
        const int j = t + q * NT;
        vm[q] = j < nvec ? vmax_of(raw[q], j) : neg_inf();
      }
      if (V > kCandMax && sampled > 0) {
        rk = rank_for(1.0f);
        theta = sample_theta<SV, NT>(vm, rk, sm);
      }
      if (t == 0) sm.cand_count = 0;
      __syncthreads();
      pc.mark(1);
#pragma unroll
      for (int q = 0; q < SV; q++) {
        const int j = t + q * NT;
        if (j < nvec && vm[q] >= theta) append_vec(raw[q], j, theta);
      }
      scalars(theta);
      scan(theta, SV * NT);
      fits = expand(theta);
    }
    pc.mark(2);
    if constexpr (kStream) {
      // fewer than k raw candidates: the threshold was too high.  Lower it here
      // (a 4x deeper rank of the sample, the row re-read while it is likely
      // still in L2), where the retry overlaps the other rows' streams, rather
      // than leaving the row to a lone fallback CTA after the finisher.
      // A list that overflowed raises theta to the tgt-th largest value it
      // buffered (every element at or above it is then in the row, so the new
      // list holds at least tgt >= k), as the fallback would, but here.
      for (int attempt = 0; attempt < kRetries && theta > neg_inf(); attempt++) {
        const bool shorted = sm.cand_count < static_cast<int>(need);
        if (!shorted && sm.cand_count <= kCandMax) break;
        float nt;
        if (shorted) {
          rk = rk * 4u;
          float vm[SV];
#pragma unroll
          for (int q = 0; q < SV; q++) {
            const int j = t + q * NT;
            vm[q] = j < nvec ? vmax_of(__ldg(vrow + j), j) : neg_inf();
          }
          nt = sample_theta<SV, NT>(vm, rk, sm);
          if (!(nt < theta)) nt = neg_inf();
        } else {
          uint32_t tk; unsigned long long b0, m0; unsigned int c0, n0;
          const unsigned int tr = static_cast<unsigned int>(tgt);
          radix_find<NT, true, false>(
              SmemSrcT<NT>{cand_y, cand_id, kCandMax, theta}, 32,
              [&](int, float y, uint32_t& key, unsigned long long& w) { key = fkey(y); w = 0; return true; },
              [&](unsigned long long, unsigned int c) { return c >= tr; }, sm, tk, b0, c0, n0, m0, 16);
          nt = key2f(tk);
          if (!(nt > theta)) break;  // ties all the way up: the fallback's full-row path decides
        }
        theta = nt;
        if (t == 0) sm.cand_count = 0;
        __syncthreads();
        scalars(theta);
        scan(theta, 0);
        fits = expand(theta);
      }
      if (t == 0) {
        a.cand_gn[b] = sm.cand_count;
        a.cand_gth[b] = theta;
      }
      return;
    }

    for (int attempt = 0;; attempt++) {
      if (need_hist && !fused) {
        const int n0 = sm.cand_count < kCandMax ? sm.cand_count : kCandMax;  // raw entries
        if (!hist.active) {
          build_hist(theta, risers);  // risers land after n0 with penalised values
        } else if (risers) {  // retry: append the risers for the new theta
          for (int s = t; s < ht; s += NT) {
            const int id = hkey[s];
            if (id < 0) continue;
            float raw = E::load(row, id);
            if (mask && !mask_allows(mask, moff + id)) raw = neg_inf();
            const float py = __int_as_float(hval[s]);
            if (!(raw >= theta) && py >= theta) {
              const int pos = atomicAdd(&sm.cand_count, 1);
              if (pos < kCandMax) { cand_y[pos] = py; cand_id[pos] = id; }
            }
          }
          __syncthreads();
        }
        for (int i = t; i < n0; i += NT) {  // raw -> penalised for history ids
          float hv;
          if (hist.find(cand_id[i], hv))
            cand_y[i] = hist_counts_only ? penalise(cand_y[i], __float_as_int(hv)) : hv;
        }
        __syncthreads();
      }
      pc.mark(3);
      const int cnt = sm.cand_count;
      const bool overflow = !fits || cnt > kCandMax;
      SmemSrcT<NT> src{cand_y, cand_id, cnt < kCandMax ? cnt : kCandMax, theta};
      const unsigned int nvalid = fused ? f_cnt : block_count_if<NT>(src, theta, sm);
      if (t == 0) atomicAdd(&a.counters[5], static_cast<unsigned long long>(nvalid));
      pc.mark(4);
      if (a.shard_out && !overflow && nvalid >= need) {  // vocab shard: emit the local record
        shard_emit<NT>(src, p, V, moff, a.shard_out + b, sm, theta > neg_inf() ? key2f(fkey(theta) - 1u) : neg_inf());
        return;
      }
      if (!overflow && nvalid >= need) {
        const bool partial = !greedy && !topk && theta > neg_inf();
        unsigned long long qrest = 0;
        if (partial) {  // exact mass of every finite element below theta (row re-read from L2)
          float ym = neg_inf();
          src.for_each([&](int, float y) { ym = fmaxf(ym, y); });
          ym = block_max<NT>(ym, sm);
          const float T = p.temperature;
          const float smax = __fdiv_rn(ym, T);
          // y <= ylim: zero mass (as in finish_row); the raw value bounds the
          // penalised one unless penalties can raise it
          const float ylim = __fmul_rn(__fsub_rn(smax, 32.0f), T);
          const bool use_lim = !(hist.active && !hist_counts_only) && fabsf(smax) < 1.0e5f;
          auto rest = [&](int v, float y) {
            if (use_lim && !(y > ylim)) return 0ull;
            float hv;
            if (hist.active && hist.find(v, hv)) y = hist_counts_only ? penalise(y, __float_as_int(hv)) : hv;
            return (y < theta && y > neg_inf()) ? qmass_le0(__fsub_rn(__fdiv_rn(y, T), smax)) : 0ull;
          };
          if (t < head) {
            float y = E::load(row, t);
            if (mask && !mask_allows(mask, moff + t)) y = neg_inf();
            qrest += rest(t, y);
          }
          if (t < V - tail0) {
            float y = E::load(row, tail0 + t);
            if (mask && !mask_allows(mask, moff + tail0 + t)) y = neg_inf();
            qrest += rest(tail0 + t, y);
          }
          for (int j = t; j < nvec; j += NT) {
            float x[EPV];
            E::unpack(__ldg(vrow + j), x);
            const uint32_t bits = mask ? mask_bits(mask, moff + head + j * EPV, EPV) : 0xffu;
#pragma unroll
            for (int e = 0; e < EPV; e++) qrest += rest(head + j * EPV + e, ((bits >> e) & 1u) ? x[e] : neg_inf());
          }
          qrest = block_sum<NT>(qrest, sm);
        }
        done = finish_cands<NT>(cand_y, cand_id, cand_e, src.n, theta, p, V, u, sm, out_id, out_prob, pc,
                                partial, qrest, 0.0f, false, fused, f_ymax, f_nymin);
        pc.mark(9);
        if (done) {
          if (t == 0) atomicAdd(&a.counters[0], 1ull);
          break;
        }
        if (t == 0) atomicAdd(&a.counters[3], 1ull);
      } else if (t == 0) {
        atomicAdd(&a.counters[overflow ? 1 : 2], 1ull);
      }
      fused = false;  // a retry rebuilds the list from raw values
      if (attempt == kRetries || theta == neg_inf()) break;
      // retry from L2 with a new threshold
      float nt;
      if (overflow) {  // the tgt-th largest of the buffered values bounds the k-th from below
        uint32_t tk; unsigned long long b0, m0; unsigned int c0, n0;
        const unsigned int tr = static_cast<unsigned int>(tgt);
        radix_find<NT, true, false>(
            src, 32,
            [&](int, float y, uint32_t& key, unsigned long long& w) { key = fkey(y); w = 0; return true; },
            [&](unsigned long long, unsigned int c) { return c >= tr; }, sm, tk, b0, c0, n0, m0, 16);
        nt = key2f(tk);
        if (!(nt > theta)) nt = neg_inf();
      } else {  // too few: a 4x deeper rank in the sample
        rk = rk * 4u;
        float vm[SV];
#pragma unroll
        for (int q = 0; q < SV; q++) {
          const int j = t + q * NT;
          vm[q] = j < nvec ? vmax_of(__ldg(vrow + j), j) : neg_inf();
        }
        nt = sample_theta<SV, NT>(vm, rk, sm);
        if (!(nt < theta)) nt = neg_inf();
      }
      theta = nt;
      if (V > kCandMax && theta == neg_inf()) break;  // nothing left but the full row
      if (t == 0) sm.cand_count = 0;
      __syncthreads();
      scalars(theta);
      scan(theta, 0);
      fits = expand(theta);
      pc.mark(10);
    }
  }
  if (!done) {
    if (t == 0) atomicAdd(&a.counters[4], 1ull);
    if (hist_counts_only) { hist.active = 0; __syncthreads(); }
    build_hist(__int_as_float(0x7f800000), true);
    GlobalSrc<DT, NT> src{row, V, head, nvec, tail0, mask, hist, moff};
    if (a.shard_out) {
      shard_emit<NT>(src, p, V, moff, a.shard_out + b, sm, neg_inf());
      return;
    }
    const bool nok_stochastic = p.temperature > 0.0f && !(p.top_k > 0 && p.top_k < V);
    if (!(nok_stochastic && finish_full<DT, NT>(src, p, u, sm, dyn, kCandMax, out_id, out_prob)))
      finish_row<NT>(src, p, V, u, false, neg_inf(), sm, out_id, out_prob);
    pc.mark(11);
  }
  if (t == 0) {
    a.out_ids[b] = out_id;
    if (a.out_probs) a.out_probs[b] = out_prob;
  }
}

template <int DT, bool kStream = false, int NT = kSampleNT>
__global__ void __launch_bounds__(NT, kStream ? kStreamCtasPerSm : (kMinCtasPerSm * kSampleNT / NT > 0 ? kMinCtasPerSm * kSampleNT / NT : 1)) sample_kernel(SampleArgs a) {
  if constexpr (kStream) {
    // launched as a programmatic dependent of whatever ran before on the stream
    // (the previous call's fallback kernel still reads the candidate buffer
    // this kernel overwrites; a producer kernel writes the logits)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // the fallback list of this launch pair starts empty
    if (a.fb_count && blockIdx.x == 0 && threadIdx.x == 0) *a.fb_count = 0;
  }
  sample_row<DT, kStream, NT>(a, blockIdx.x);
}

// The rows the warp finisher left (a.fb_rows[0 .. *a.fb_count)): CTA i takes
// entry i; the grid covers every row of the call, and CTAs past the count exit
// at once.  (A grid-stride loop over a few CTAs per SM spilled five times as
// much and made rows without top-k 1.4-1.7x slower.)
#ifndef TG_LIST_MINB
#define TG_LIST_MINB TG_MIN_CTAS
#endif
template <int DT>
__global__ void __launch_bounds__(kSampleNT, TG_LIST_MINB) sample_list_kernel(SampleArgs a) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the finisher's list (programmatic launch)
  if (static_cast<int>(blockIdx.x) >= *a.fb_count) return;
  sample_row<DT, false, kSampleNT>(a, a.fb_rows[blockIdx.x]);
}

// ---- vocab-sharded mode, merge half ---------------------------------------
struct MergeArgs {
  const tg_shard_record* rec;  // [nshards][batch]
  int32_t nshards;
  int32_t batch;
  int32_t full_vocab;
  const tg_row_params* params;
  const float* uniforms;
  int32_t* out_ids;
  float* out_probs;
  uint32_t* status;
};

struct RecSrc {  // every entry of one row's records
  const tg_shard_record* rec;
  int nshards, batch, row;
  template <class F>
  __device__ __forceinline__ void for_each(F&& f) const {
    for (int r = 0; r < nshards; r++) {
      const tg_shard_record* x = rec + static_cast<int64_t>(r) * batch + row;
      const int c = x->count;
      for (int i = threadIdx.x; i < c; i += kSampleNT) f(x->cand[i].id, x->cand[i].value);
    }
  }
};

// One CTA per row.  The union of the shards' local top-k survivors holds every
// element >= the global k-th value, so the global k-th is found over the union
// and stages (b)-(e) run on the entries >= it, exactly as in sample_kernel.
__global__ void __launch_bounds__(kSampleNT) sample_merge_kernel(MergeArgs m) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ BlockScratch sm;
  const int b = blockIdx.x;
  const int t = threadIdx.x;
  float* cand_y = reinterpret_cast<float*>(dyn);
  int* cand_id = reinterpret_cast<int*>(dyn + kCandMax * 4);
  float* cand_e = reinterpret_cast<float*>(dyn + kCandMax * 8);
  const tg_row_params p = m.params[b];
  const float u = m.uniforms ? m.uniforms[b] : 0.0f;
  bool bad = false;
  float absent = neg_inf();  // no value missing from the union exceeds this
  for (int r = 0; r < m.nshards; r++) {
    const tg_shard_record* x = m.rec + static_cast<int64_t>(r) * m.batch + b;
    bad |= x->count < 0 || x->flags != 0;
    absent = fmaxf(absent, x->absent_max);
  }
  int out_id = -1;
  float out_prob = 0.0f;
  RecSrc src{m.rec, m.nshards, m.batch, b};
  if (!bad) {
    const bool greedy = !(p.temperature > 0.0f);
    float kth = neg_inf();
    if (!greedy && p.top_k < m.full_vocab) {
      uint32_t kkey; unsigned long long b0, m0; unsigned int c0, n0;
      const unsigned int k = static_cast<unsigned int>(p.top_k);
      auto kw = [&](int, float y, uint32_t& key, unsigned long long& w) {
        if (!(y > neg_inf())) return false;
        key = fkey(y); w = 0; return true;
      };
      auto rc = [&](unsigned long long, unsigned int c) { return c >= k; };
      radix_find<kSampleNT, true, false, RecSrc, decltype(kw), decltype(rc), true>(src, 32, kw, rc, sm, kkey, b0, c0, n0, m0);
      kth = key2f(kkey);
    }
    if (t == 0) sm.sn = 0;
    __syncthreads();
    src.for_each([&](int id, float y) {
      if (y >= kth && y > neg_inf()) {
        const int pos = atomicAdd(&sm.sn, 1);
        if (pos < kCandMax) { cand_y[pos] = y; cand_id[pos] = id; }
      }
    });
    __syncthreads();
    const int n = sm.sn;
    __syncthreads();
    if (n > kCandMax) {
      bad = true;
    } else {
      PhaseClock pc;
      bad = !finish_cands(cand_y, cand_id, cand_e, n, kth, p, m.full_vocab, u, sm, out_id, out_prob, pc,
                          false, 0ull, absent, true);
    }
  }
  if (t == 0) {
    if (bad) { out_id = -1; out_prob = 0.0f; atomicOr(m.status, 4u); }
    m.out_ids[b] = out_id;
    if (m.out_probs) m.out_probs[b] = out_prob;
  }
}

}  // namespace tg
