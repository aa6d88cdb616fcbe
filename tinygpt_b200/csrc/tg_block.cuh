// tg_block.cuh -- CTA-wide building blocks: reductions, a warp-aggregated
// candidate append, and a weighted MSB-first radix search.
#pragma once

#include "tg_common.cuh"

namespace tg {

constexpr unsigned kFull = 0xffffffffu;
// Largest element count of a wide mass histogram: its 15-bit limb sums stay below 2^32.
constexpr int kWideMassN = 1 << 16;

__device__ __forceinline__ unsigned long long radix_mass_of(const unsigned int (&l)[4][256], int bin) {
  return static_cast<unsigned long long>(l[0][bin]) + (static_cast<unsigned long long>(l[1][bin]) << 11) +
         (static_cast<unsigned long long>(l[2][bin]) << 22) + (static_cast<unsigned long long>(l[3][bin]) << 33);
}

// Barrier of the NT threads of a CTA-wide stage: __syncthreads when BAR is 0,
// else the named barrier BAR over NT threads (a warp-specialized CTA whose
// other warps run other work).
template <int NT, int BAR>
__device__ __forceinline__ void bsync() {
  if constexpr (BAR == 0) {
    __syncthreads();
  } else {
    asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
  }
}

struct __align__(16) BlockScratch {
  // Mass histograms are kept as 32-bit limbs of the 64-bit sums: shared-memory
  // 32-bit atomic adds are native, 64-bit ones are compare-and-swap loops that
  // serialise when lanes hit the same bin.
  union {
    struct {
      unsigned int hml[4][256];  // radix mass, 11-bit limbs (sums of up to 2^20 masses <= 2^44)
      unsigned int hcnt[256];
      unsigned int hfine[256];  // elements whose key has non-zero low 16 bits (kEarly16)
    };
    unsigned int hc[2048];        // wide count histogram (hist_round)
    unsigned int hm3[3][1024];    // wide mass histogram, 15-bit limbs (at most kWideMassN masses)
  };
  unsigned long long red_u64[32];
  float red_f[32];
  int red_i[32];
  unsigned long long sel_before;
  unsigned long long sel_mass;
  unsigned int sel_bin;
  unsigned int sel_cbefore;
  unsigned int sel_cnt;
  int cand_count;
  // small list for warp-level resolution of one histogram bin
  unsigned long long sk[32];
  unsigned long long sw[32];
  int sid[32];
  int sn;
  float red_f2[32];
};

// Reductions need only the red_* fields: S is BlockScratch or ReduceScratch.
struct ReduceScratch {
  unsigned long long red_u64[32];
  float red_f[32];
  int red_i[32];
  float red_f2[32];
};

template <int NT, class S, int BAR = 0>
__device__ __forceinline__ float block_max(float v, S& sm) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  if ((threadIdx.x & 31) == 0) sm.red_f[threadIdx.x >> 5] = v;
  bsync<NT, BAR>();
  float r = sm.red_f[0];
#pragma unroll
  for (int i = 1; i < NT / 32; i++) r = fmaxf(r, sm.red_f[i]);
  bsync<NT, BAR>();
  return r;
}

// Two maxima with one pair of barriers.
template <int NT, class S, int BAR = 0>
__device__ __forceinline__ void block_max2(float& a, float& b, S& sm) {
  for (int o = 16; o > 0; o >>= 1) {
    a = fmaxf(a, __shfl_xor_sync(kFull, a, o));
    b = fmaxf(b, __shfl_xor_sync(kFull, b, o));
  }
  if ((threadIdx.x & 31) == 0) { sm.red_f[threadIdx.x >> 5] = a; sm.red_f2[threadIdx.x >> 5] = b; }
  bsync<NT, BAR>();
  a = sm.red_f[0];
  b = sm.red_f2[0];
#pragma unroll
  for (int i = 1; i < NT / 32; i++) { a = fmaxf(a, sm.red_f[i]); b = fmaxf(b, sm.red_f2[i]); }
  bsync<NT, BAR>();
}

template <int NT, class S>
__device__ __forceinline__ unsigned long long block_sum(unsigned long long v, S& sm) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  if ((threadIdx.x & 31) == 0) sm.red_u64[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long r = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; i++) r += sm.red_u64[i];
  __syncthreads();
  return r;
}

template <int NT, class S>
__device__ __forceinline__ unsigned int block_max_u32(unsigned int v, S& sm) {
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(kFull, v, o));
  if ((threadIdx.x & 31) == 0) sm.red_i[threadIdx.x >> 5] = static_cast<int>(v);
  __syncthreads();
  unsigned int r = static_cast<unsigned int>(sm.red_i[0]);
#pragma unroll
  for (int i = 1; i < NT / 32; i++) r = max(r, static_cast<unsigned int>(sm.red_i[i]));
  __syncthreads();
  return r;
}

// Max y, then the smallest id holding it.  Returns via references.
template <int NT, class S>
__device__ __forceinline__ void block_argmax(float& y, int& id, S& sm) {
  for (int o = 16; o > 0; o >>= 1) {
    const float oy = __shfl_xor_sync(kFull, y, o);
    const int oi = __shfl_xor_sync(kFull, id, o);
    if (oy > y || (oy == y && oi < id)) { y = oy; id = oi; }
  }
  if ((threadIdx.x & 31) == 0) {
    sm.red_f[threadIdx.x >> 5] = y;
    sm.red_i[threadIdx.x >> 5] = id;
  }
  __syncthreads();
  y = sm.red_f[0];
  id = sm.red_i[0];
#pragma unroll
  for (int i = 1; i < NT / 32; i++) {
    const float oy = sm.red_f[i];
    const int oi = sm.red_i[i];
    if (oy > y || (oy == y && oi < id)) { y = oy; id = oi; }
  }
  __syncthreads();
}

// Exclusive prefix sum of one u64 per thread in thread order; also the total.
template <int NT, class S, int BAR = 0>
__device__ __forceinline__ unsigned long long block_excl_scan(unsigned long long v,
                                                              unsigned long long& total,
                                                              S& sm) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  unsigned long long incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long n = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) sm.red_u64[w] = incl;
  bsync<NT, BAR>();
  unsigned long long before = 0;
  total = 0;
#pragma unroll
  for (int i = 0; i < NT / 32; i++) {
    const unsigned long long s = sm.red_u64[i];
    if (i < w) before += s;
    total += s;
  }
  bsync<NT, BAR>();
  return before + incl - v;
}

// Append the elements flagged in `hits` (bit e = x[e], token e0+e) to the
// candidate arrays.  Must be called by all 32 lanes of the warp.
template <int N, int CMAX>
__device__ __forceinline__ void warp_append(uint32_t hits, const float* x, int e0, float* cy,
                                            int* cid, int* counter) {
  const int lane = threadIdx.x & 31;
  const int cnt = __popc(hits);
  int incl = cnt;
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += n;
  }
  const int total = __shfl_sync(kFull, incl, 31);
  if (total == 0) return;
  int base = 0;
  if (lane == 31) base = atomicAdd(counter, total);
  base = __shfl_sync(kFull, base, 31);
  int pos = base + incl - cnt;
#pragma unroll
  for (int e = 0; e < N; e++) {
    if ((hits >> e) & 1u) {
      if (pos < CMAX) { cy[pos] = x[e]; cid[pos] = e0 + e; }
      pos++;
    }
  }
}

// One histogram round with NB bins (NB a multiple of NT) and an all-thread scan.
// binw(i, y, bin, w) -> bool: whether the element takes part and its bin, given
// in scan order (the caller maps descending keys to ascending bins).  Returns
// the first bin at which reached(cumulative weight) holds, the weight before it
// and the weight in it.  Weights are counts (kMass = false) or u64 masses.
// reached(0) must be false and reached(total) true.
struct HistSel {
  int bin;
  unsigned long long before;
  unsigned long long in_bin;
};

// hist_zero + (caller's pass calling hist_put) + hist_scan is a hist_round
// whose accumulation rides inside another pass over the data.  The caller
// synchronizes between hist_zero and the first hist_put.
template <int NT, int NB, bool kMass>
__device__ __forceinline__ void hist_zero(BlockScratch& sm) {
  static_assert(NB % NT == 0, "bins must be a multiple of the block");
  static_assert(kMass ? NB <= 1024 : NB <= 2048, "histogram does not fit");
  constexpr int P = NB / NT;
#pragma unroll
  for (int j = 0; j < P; j++) {
    if (kMass) {
      sm.hm3[0][threadIdx.x * P + j] = 0u;
      sm.hm3[1][threadIdx.x * P + j] = 0u;
      sm.hm3[2][threadIdx.x * P + j] = 0u;
    }
    else sm.hc[threadIdx.x * P + j] = 0u;
  }
  if (threadIdx.x == 0) sm.sel_bin = 0xffffffffu;
}

template <bool kMass>
__device__ __forceinline__ void hist_put(BlockScratch& sm, int bin, unsigned long long w) {
  if (kMass) {  // w <= 2^44
    atomicAdd(&sm.hm3[0][bin], static_cast<unsigned>(w & 0x7fffu));
    atomicAdd(&sm.hm3[1][bin], static_cast<unsigned>((w >> 15) & 0x7fffu));
    atomicAdd(&sm.hm3[2][bin], static_cast<unsigned>(w >> 30));
  } else {
    atomicAdd(&sm.hc[bin], 1u);
  }
}

template <int NT, int NB, bool kMass, class Reached, int BAR = 0>
__device__ HistSel hist_scan(Reached reached, BlockScratch& sm) {
  constexpr int P = NB / NT;
  const int t = threadIdx.x;
  bsync<NT, BAR>();
  unsigned long long v[P];
  unsigned long long loc = 0;
#pragma unroll
  for (int j = 0; j < P; j++) {
    const int b = t * P + j;
    v[j] = kMass ? static_cast<unsigned long long>(sm.hm3[0][b]) + (static_cast<unsigned long long>(sm.hm3[1][b]) << 15) +
                       (static_cast<unsigned long long>(sm.hm3[2][b]) << 30)
                 : static_cast<unsigned long long>(sm.hc[b]);
    loc += v[j];
  }
  unsigned long long tot;
  const unsigned long long bef = block_excl_scan<NT, BlockScratch, BAR>(loc, tot, sm);
  if (!reached(bef) && reached(bef + loc)) {
    unsigned long long c = bef;
#pragma unroll
    for (int j = 0; j < P; j++) {
      if (reached(c + v[j])) {
        sm.sel_bin = t * P + j;
        sm.sel_before = c;
        sm.sel_mass = v[j];
        break;
      }
      c += v[j];
    }
  }
  bsync<NT, BAR>();
  HistSel r{static_cast<int>(sm.sel_bin), sm.sel_before, sm.sel_mass};  // bin -1: not reached
  bsync<NT, BAR>();
  return r;
}

template <int NT, int NB, bool kMass, class Src, class BinW, class Reached, int BAR = 0>
__device__ HistSel hist_round(const Src& src, BinW binw, Reached reached, BlockScratch& sm) {
  hist_zero<NT, NB, kMass>(sm);
  bsync<NT, BAR>();
  src.for_each([&](int i, float y) {
    int bin;
    unsigned long long w;
    if (binw(i, y, bin, w)) hist_put<kMass>(sm, bin, w);
  });
  return hist_scan<NT, NB, kMass, Reached, BAR>(reached, sm);
}

// Collect the elements for which member(i, y, key, w, id) holds into the small
// list (first 32 kept); returns how many there were.
template <int NT, class Src, class Member>
__device__ int collect_small(const Src& src, Member member, BlockScratch& sm) {
  if (threadIdx.x == 0) sm.sn = 0;
  __syncthreads();
  src.for_each([&](int i, float y) {
    unsigned long long key, w;
    int id;
    if (!member(i, y, key, w, id)) return;
    const int pos = atomicAdd(&sm.sn, 1);
    if (pos < 32) { sm.sk[pos] = key; sm.sw[pos] = w; sm.sid[pos] = id; }
  });
  __syncthreads();
  const int n = sm.sn;
  __syncthreads();
  return n;
}

// Warp 0: sort the small list (n <= 32) by key ascending, then the inclusive
// running weight from `before`; the first position where reached() holds.
// Outputs (valid in warp 0): that position's key, weight and id, and whether
// any position reached.
template <class Reached>
__device__ __forceinline__ bool warp_sorted_pick(int n, unsigned long long before, Reached reached,
                                                 const BlockScratch& sm, unsigned long long& key,
                                                 unsigned long long& w, int& id) {
  const int lane = threadIdx.x & 31;
  unsigned long long k = lane < n ? sm.sk[lane] : ~0ull;
  unsigned long long x = lane < n ? sm.sw[lane] : 0ull;
  int d = lane < n ? sm.sid[lane] : 0x7fffffff;
  for (int size = 2; size <= 32; size <<= 1) {
    for (int j = size >> 1; j > 0; j >>= 1) {
      const unsigned long long ok = __shfl_xor_sync(kFull, k, j);
      const unsigned long long ox = __shfl_xor_sync(kFull, x, j);
      const int od = __shfl_xor_sync(kFull, d, j);
      const bool up = (lane & size) == 0;
      const bool lower = (lane & j) == 0;
      const bool take = (lower == up) ? (ok < k) : (ok > k);
      if (take) { k = ok; x = ox; d = od; }
    }
  }
  unsigned long long incl = x;
  for (int o = 1; o < 32; o <<= 1) {
    const unsigned long long v = __shfl_up_sync(kFull, incl, o);
    if (lane >= o) incl += v;
  }
  const unsigned hit = __ballot_sync(kFull, lane < n && reached(before + incl));
  const int src = hit ? __ffs(hit) - 1 : (n > 0 ? n - 1 : 0);
  key = __shfl_sync(kFull, k, src);
  w = __shfl_sync(kFull, x, src);
  id = __shfl_sync(kFull, d, src);
  return hit != 0;
}

// Histogram update aggregated over the lanes of a warp that hit the same bin
// (one shared atomic per distinct bin per warp instead of one per lane).
template <bool kMass>
__device__ __forceinline__ void hist_add(BlockScratch& sm, uint32_t d, unsigned long long w) {
  const unsigned act = __activemask();
  const unsigned peers = __match_any_sync(act, d);
  unsigned l[4] = {0u, 0u, 0u, 0u};
  if (kMass) {  // w <= 2^44: four 11-bit limbs, each summed over the peers
#pragma unroll
    for (int i = 0; i < 4; i++) l[i] = __reduce_add_sync(peers, static_cast<unsigned>((w >> (11 * i)) & (i == 3 ? 0xfffu : 0x7ffu)));
  }
  if ((threadIdx.x & 31) == __ffs(peers) - 1) {
    atomicAdd(&sm.hcnt[d], static_cast<unsigned>(__popc(peers)));
    if (kMass) {
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (l[i]) atomicAdd(&sm.hml[i][d], l[i]);
    }
  }
}

// Weighted MSB-first radix search over the elements a Source yields.
//
// keyw(id, y, key, w) -> bool: whether the element takes part, its key
// (nbits wide) and weight.  Digits are scanned in descending key order when
// kDesc, ascending otherwise, accumulating (mass, count) from the keys already
// passed; the result is the key of the element at which reached(mass, count)
// first holds, including that key's whole bin.  Outputs: the key, the mass and
// count strictly before it in scan order, and the mass and count of elements
// with exactly that key.
// Rounds stop once the bits above `min_shift` are resolved (the low bits of
// key_out are then zero: the search is approximate below that resolution).
// kEarly16: stop after the top 16 bits when no element of the selected bin has
// non-zero low 16 bits (all of them then share the key exactly -- the common
// case for bf16 logits).
template <int NT, bool kDesc, bool kMass, class Src, class KeyW, class Reached, bool kEarly16 = false>
__device__ void radix_find(const Src& src, int nbits, KeyW keyw, Reached reached,
                           BlockScratch& sm, uint32_t& key_out, unsigned long long& before_out,
                           unsigned int& cbefore_out, unsigned int& cnt_out,
                           unsigned long long& mass_out, int min_shift = 0) {
  uint32_t prefix = 0, pmask = 0;
  unsigned long long before = 0;
  unsigned int cbefore = 0;
  unsigned int bcnt = 0;
  unsigned long long bmass = 0;
  int shift = nbits;
  while (shift > min_shift) {
    const int width = shift >= 8 ? 8 : shift;
    shift -= width;
    const uint32_t dmask = (1u << width) - 1u;
    const bool fine_round = kEarly16 && shift == 16;
    for (int i = threadIdx.x; i < 256; i += NT) {
      sm.hml[0][i] = 0u; sm.hml[1][i] = 0u; sm.hml[2][i] = 0u; sm.hml[3][i] = 0u;
      sm.hcnt[i] = 0u;
      if (fine_round) sm.hfine[i] = 0u;
    }
    __syncthreads();
    src.for_each([&](int id, float y) {
      uint32_t key;
      unsigned long long w;
      if (!keyw(id, y, key, w)) return;
      if ((key & pmask) != prefix) return;
      hist_add<kMass>(sm, (key >> shift) & dmask, w);
      if (fine_round && (key & 0xffffu)) atomicAdd(&sm.hfine[(key >> shift) & dmask], 1u);
    });
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      const int nb = 1 << width;
      const int per = (nb + 31) >> 5;
      unsigned long long lm = 0;
      unsigned int lc = 0;
      for (int q = 0; q < per; q++) {
        const int p = lane * per + q;
        if (p < nb) {
          const int bin = kDesc ? nb - 1 - p : p;
          lm += kMass ? radix_mass_of(sm.hml, bin) : 0ull;
          lc += sm.hcnt[bin];
        }
      }
      unsigned long long em = lm;
      unsigned int ec = lc;
      for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long tm = __shfl_up_sync(kFull, em, o);
        const unsigned int tc = __shfl_up_sync(kFull, ec, o);
        if (lane >= o) { em += tm; ec += tc; }
      }
      em -= lm;
      ec -= lc;
      unsigned long long cm = before + em;
      unsigned int cc = cbefore + ec;
      int found = -1, last = -1;
      unsigned long long fb = 0, lb = 0;
      unsigned int fcb = 0, lcb = 0;
      for (int q = 0; q < per; q++) {
        const int p = lane * per + q;
        if (p < nb) {
          const int bin = kDesc ? nb - 1 - p : p;
          const unsigned long long m = kMass ? radix_mass_of(sm.hml, bin) : 0ull;
          const unsigned int c = sm.hcnt[bin];
          if (c > 0) {
            if (found < 0 && reached(cm + m, cc + c)) { found = bin; fb = cm; fcb = cc; }
            last = bin; lb = cm; lcb = cc;
          }
          cm += m;
          cc += c;
        }
      }
      const unsigned bal = __ballot_sync(kFull, found >= 0);
      if (bal) {
        if (lane == __ffs(bal) - 1) {
          sm.sel_bin = found; sm.sel_before = fb; sm.sel_cbefore = fcb;
        }
      } else {  // target beyond the total (defensive): take the last non-empty bin
        const unsigned bl = __ballot_sync(kFull, last >= 0);
        if (bl && lane == 31 - __clz(bl)) {
          sm.sel_bin = last; sm.sel_before = lb; sm.sel_cbefore = lcb;
        } else if (!bl && lane == 0) {
          sm.sel_bin = 0; sm.sel_before = before; sm.sel_cbefore = cbefore;
        }
      }
      __syncwarp();
      if (lane == 0) {
        sm.sel_cnt = sm.hcnt[sm.sel_bin];
        sm.sel_mass = kMass ? radix_mass_of(sm.hml, sm.sel_bin) : 0ull;
      }
    }
    __syncthreads();
    const uint32_t bin = sm.sel_bin;
    before = sm.sel_before;
    cbefore = sm.sel_cbefore;
    bcnt = sm.sel_cnt;
    bmass = sm.sel_mass;
    prefix |= bin << shift;
    pmask |= dmask << shift;
    const bool exact = fine_round && sm.hfine[bin] == 0u;
    __syncthreads();
    if (exact) break;
  }
  key_out = prefix;
  before_out = before;
  cbefore_out = cbefore;
  cnt_out = bcnt;
  mass_out = bmass;
}

}  // namespace tg
