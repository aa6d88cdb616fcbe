// tg_fused.cuh -- the streaming and finishing halves of a large tg_sample call
// in ONE persistent kernel, so that the finishing stages of earlier rows run
// while later rows stream from HBM.
//
// One CTA per SM; CTA c takes rows c, c + grid, c + 2 grid, ...  Its warps:
//   * a producer warp (one elected lane) streams each row's 16-byte-aligned
//     body into a shared-memory ring of 16 KB stages with 1-D bulk copies
//     (cp.async.bulk, completion on an mbarrier per stage; the source is this
//     GPU's own logits and no copy is multicast), so the bytes in flight are
//     held by shared memory, not by registers;
//   * 8 filter warps (256 threads) compute the row's threshold theta from its
//     first stage (the same sample as sample_kernel: the first 4 vectors of
//     each of 256 threads), then test every 128-bit vector of every stage
//     against theta and append the elements >= theta to the row's candidate
//     list, which lives in a shared-memory slot;
//   * finisher groups of 4 warps each take a published slot and run stages
//     (a)-(e) on it (grp_finish_row, tg_finish_warp.cuh), writing the id.
// Rows the finishers do not take leave their raw list in global memory and go
// to the fallback list (sample_list_kernel runs them afterwards), exactly as
// in the two-kernel mode; rows that are not streamed at all (top-k > 1024,
// plain temperature, a bad grammar state) go there with cand_gn = -1.
//
// Every wait is bounded (kFuWaitLimit polls).  A wait that runs out sets
// device status bit 3 and the CTA's abort flag; every role polls the flag and
// leaves, the producer first waiting (bounded) for the copies it issued.
#pragma once

#include "tg_finish_warp.cuh"

namespace tg {

constexpr int kFuFilterNT = kSampleNT;                   // 8 filter warps
constexpr int kFuChunkVecs = kSampleVecs * kFuFilterNT;  // 1024 vectors: the sample is stage 0
constexpr int kFuChunkBytes = kFuChunkVecs * 16;         // 16 KB per stage
constexpr int kFuG = 4;                                  // warps per finisher group
constexpr int kFuMaxStages = 8;
constexpr int kFuMaxSlots = 6;
constexpr int kFuProducerTid = kFuFilterNT;              // warp 8
constexpr int kFuFinTid0 = kFuFilterNT + 32;             // finisher groups from warp 9
constexpr unsigned kFuWaitLimit = 1u << 24;
constexpr int kFuSmem = 227 * 1024 - 1024;               // dynamic shared memory (static: FusedCtl)
constexpr int kFuBarFilter = 1;                          // named barrier of the filter warps
constexpr int kFuBarFin0 = 2;                            // finisher group i: 2 + i

struct FusedCfg {
  int stages;       // ring stages (<= kFuMaxStages)
  int slots;        // candidate-list slots (<= kFuMaxSlots)
  int groups;       // finisher groups (= slots - 1)
  int off_slots;    // dynamic shared-memory offsets
  int off_filter;
  int off_rings;
  int off_fin;
  int debug;        // diagnostics (bit 0: finishers skip every row)
};

__host__ __device__ __forceinline__ size_t fused_smem(int stages, int slots, int groups, int ht_log2, FusedCfg* c) {
  size_t o = static_cast<size_t>(stages) * kFuChunkBytes;
  const size_t slots_off = o;
  o += static_cast<size_t>(slots) * kCandMax * 8;
  const size_t filt = o;
  o += (sizeof(BlockScratch) + 127) & ~size_t(127);
  const size_t rings = o;
  o += static_cast<size_t>(kFuFilterNT / 32) * kRing * 20;
  o = (o + 127) & ~size_t(127);
  const size_t fin = o;
  o += static_cast<size_t>(groups) * grp_fin_bytes(ht_log2);
  if (c) {
    c->stages = stages;
    c->slots = slots;
    c->groups = groups;
    c->off_slots = static_cast<int>(slots_off);
    c->off_filter = static_cast<int>(filt);
    c->off_rings = static_cast<int>(rings);
    c->off_fin = static_cast<int>(fin);
  }
  return o;
}

struct FusedCtl {
  uint64_t full[kFuMaxStages];
  uint64_t empty[kFuMaxStages];
  int slot_pub[kFuMaxSlots];    // q + 1 once this CTA's q-th streamed row is in the slot
  int slot_free[kFuMaxSlots];   // times the slot was released
  int slot_row[kFuMaxSlots];
  int slot_n[kFuMaxSlots];
  float slot_theta[kFuMaxSlots];
  int claim;                    // next streamed row a finisher group claims
  int total;                    // streamed rows of this CTA (valid once done != 0)
  int done;
  int abort;
  int gq[16];                   // the row index each finisher group claimed
};

__device__ __forceinline__ int ld_acquire_cta(const int* p) {
  int v;
  asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_cta(int* p, int v) {
  asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

// Bounded wait for the completion of the phase with the given parity.
__device__ __forceinline__ bool mbar_wait_parity(uint64_t* bar, uint32_t parity, const int* abort) {
  for (unsigned it = 0; it < kFuWaitLimit; it++) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 1023u) == 1023u && *reinterpret_cast<const volatile int*>(abort)) return false;
  }
  return false;
}

// Whether the fused kernel streams row b (sample_row's `fast` rows with a
// valid grammar state); the same predicate runs in the producer and the
// filter warps so both walk the same stages.
__device__ __forceinline__ bool fused_streams(const SampleArgs& a, int b) {
  const tg_row_params p = a.params[b];
  const int V = a.vocab;
  const bool greedy = !(p.temperature > 0.0f);
  const bool topk = p.top_k > 0 && p.top_k < V;
  const bool truncated = p.top_p < 1.0f || p.min_p > 0.0f;
  const bool fast = greedy || (topk && p.top_k <= kFastMaxK) || (!topk && truncated);
  if (!fast) return false;
  if (a.mask_table && a.state_id && a.state_id[b] >= a.num_states) return false;
  return true;
}

template <int DT>
__device__ __forceinline__ void row_geometry(const SampleArgs& a, int b, const char*& row, int& head, int& nvec,
                                             int& tail0) {
  using E = Elt<DT>;
  row = reinterpret_cast<const char*>(a.logits) + b * a.row_stride * E::kSize;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(row);
  head = static_cast<int>(((16u - (addr & 15u)) & 15u) / E::kSize);
  if (head > a.vocab) head = a.vocab;
  nvec = (a.vocab - head) / E::kEPV;
  tail0 = head + nvec * E::kEPV;
}

// Diagnostic build only (-DTG_PHASE_TIMING): cycles of one thread per role
// added to g_phase_cycles[i].
__device__ __forceinline__ void fu_add(int i, long long c) {
#ifdef TG_PHASE_TIMING
  atomicAdd(&g_phase_cycles[i], static_cast<unsigned long long>(c));
#else
  (void)i;
  (void)c;
#endif
}

__device__ __forceinline__ void fused_fallback(const SampleArgs& a, int b) {
  const int pos = atomicAdd(a.fb_count, 1);
  a.fb_rows[pos] = b;
}

template <int DT>
__global__ void __launch_bounds__(kFuFinTid0 + 4 * 32 * kFuG, 1) sample_fused_kernel(SampleArgs a, FusedCfg cfg) {
  using E = Elt<DT>;
  constexpr int EPV = E::kEPV;
  constexpr int NT = kFuFilterNT;
  // a vector of -inf (outside the row)
  const uint4 kNegVec = DT == 1 ? make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u)
                                : make_uint4(0xff800000u, 0xff800000u, 0xff800000u, 0xff800000u);
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ FusedCtl ctl;
  const int tid = threadIdx.x;
  const int S = cfg.stages, NS = cfg.slots;
  unsigned char* ring = dyn;
  unsigned char* slots = dyn + cfg.off_slots;

  if (tid == 0) {
    for (int i = 0; i < S; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&ctl.full[i])) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&ctl.empty[i])), "r"(NT / 32) : "memory");
    }
    for (int i = 0; i < kFuMaxSlots; i++) { ctl.slot_pub[i] = 0; ctl.slot_free[i] = 0; }
    ctl.claim = 0;
    ctl.total = 0;
    ctl.done = 0;
    ctl.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  auto fail = [&]() {
    ctl.abort = 1;
    atomicOr(a.status, 8u);
  };

  if (tid >= kFuProducerTid && tid < kFuFinTid0) {
    // ---------------- producer ----------------
    if (tid != kFuProducerTid) return;
    unsigned g = 0;  // stages issued
    bool ok = true;
    for (int b = blockIdx.x; ok && b < a.batch; b += gridDim.x) {
      if (!fused_streams(a, b)) continue;
      const char* row;
      int head, nvec, tail0;
      row_geometry<DT>(a, b, row, head, nvec, tail0);
      const char* vrow = row + head * E::kSize;
      for (int c = 0; c * kFuChunkVecs < nvec; c++, g++) {
        const int st = static_cast<int>(g % S);
        if (g >= static_cast<unsigned>(S) && !mbar_wait_parity(&ctl.empty[st], ((g / S) - 1u) & 1u, &ctl.abort)) {
          ok = false;
          break;
        }
        const int nv = min(kFuChunkVecs, nvec - c * kFuChunkVecs);
        const uint32_t bytes = static_cast<uint32_t>(nv) * 16u;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(&ctl.full[st])),
                     "r"(bytes)
                     : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(ring + static_cast<size_t>(st) * kFuChunkBytes)),
            "l"(vrow + static_cast<int64_t>(c) * kFuChunkBytes), "r"(bytes), "r"(smem_u32(&ctl.full[st]))
            : "memory");
      }
    }
    if (!ok) fail();
    // the copies issued last must have landed before the CTA may exit
    const unsigned first = g > static_cast<unsigned>(S) ? g - S : 0u;
    for (unsigned q = first; q < g; q++) {
      uint64_t* bar = &ctl.full[q % S];
      for (unsigned it = 0; it < kFuWaitLimit; it++) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"((q / S) & 1u)
            : "memory");
        if (done) break;
      }
    }
    return;
  }

  if (tid >= kFuFinTid0) {
    // ---------------- finisher groups ----------------
    const int ft = tid - kFuFinTid0;
    const Grp<kFuG> g{ft / (32 * kFuG), ft % (32 * kFuG), (ft % (32 * kFuG)) >> 5, ft & 31,
                      kFuBarFin0 + ft / (32 * kFuG)};
    if (g.id >= cfg.groups) return;
    unsigned char* scratch = dyn + cfg.off_fin + static_cast<size_t>(g.id) * grp_fin_bytes(a.ht_log2);
    for (;;) {
      const long long c0 = clock64();
      if (g.gt == 0) {
        int q = atomicAdd(&ctl.claim, 1);
        const int s = q % NS;
        bool ready = false;
        for (unsigned it = 0; it < kFuWaitLimit; it++) {
          if (ld_acquire_cta(&ctl.slot_pub[s]) == q + 1) { ready = true; break; }
          if (ld_acquire_cta(&ctl.done) && q >= ld_acquire_cta(&ctl.total)) break;
          if (*reinterpret_cast<volatile int*>(&ctl.abort)) break;
          __nanosleep(256);  // leave the issue slots to the filter warps
        }
        if (!ready) {
          if (!ld_acquire_cta(&ctl.done) && !*reinterpret_cast<volatile int*>(&ctl.abort)) fail();
          q = -1;
        }
        ctl.gq[g.id] = q;
      }
      g.sync();
      const int q = ctl.gq[g.id];
      g.sync();
      const long long c1 = clock64();
      if (g.gt == 0) fu_add(27, c1 - c0);  // 27: finisher waits for a published row
      if (q < 0) return;
      const int s = q % NS;
      const int b = ctl.slot_row[s];
      const int n = ctl.slot_n[s];
      const float theta = ctl.slot_theta[s];
      float* ly = reinterpret_cast<float*>(slots + static_cast<size_t>(s) * kCandMax * 8);
      int* lid = reinterpret_cast<int*>(ly + kCandMax);
      bool ok = false;
      if (cfg.debug & 1) {  // diagnostics: the finishers leave every row to the fallback
        if (g.gt == 0) a.cand_gn[b] = -1;
      } else if (grp_can_take(a, b, n, theta)) {
        ok = grp_finish_row<kFuG, false>(g, a, b, n, theta, scratch, ly, lid);
        if (!ok && g.gt == 0) a.cand_gn[b] = -1;  // the list was modified: the fallback streams the row
      } else {  // raw list out to global memory for the fallback's candidate path
        const int m = n < kCandMax ? n : kCandMax;
        float* gy = a.cand_gy + static_cast<int64_t>(b) * kCandMax;
        int* gid = a.cand_gid + static_cast<int64_t>(b) * kCandMax;
        for (int i = g.gt; i < m; i += 32 * kFuG) { gy[i] = ly[i]; gid[i] = lid[i]; }
        if (g.gt == 0) { a.cand_gn[b] = n; a.cand_gth[b] = theta; }
      }
      g.sync();  // every thread is done with the slot
      if (g.gt == 0) fu_add(28, clock64() - c1);  // 28: finishing
      if (g.gt == 0) {
        if (ok) {
          atomicAdd(&a.counters[0], 1ull);
          atomicAdd(&a.counters[6], 1ull);
        } else {
          fused_fallback(a, b);
        }
        st_release_cta(&ctl.slot_free[s], ctl.slot_free[s] + 1);
      }
    }
  }

  // ---------------- filter warps (tid < 256) ----------------
  const int t = tid;
  const int lane = t & 31, warp = t >> 5;
  const unsigned lt = (1u << lane) - 1u;
  uint4* rdata = reinterpret_cast<uint4*>(dyn + cfg.off_rings) + warp * kRing;
  int* ridx = reinterpret_cast<int*>(reinterpret_cast<uint4*>(dyn + cfg.off_rings) + (NT / 32) * kRing) + warp * kRing;
  BlockScratch& sm = *reinterpret_cast<BlockScratch*>(dyn + cfg.off_filter);
  auto fbar = [&]() { bsync<NT, kFuBarFilter>(); };
  const int V = a.vocab;
  unsigned g = 0;  // stages consumed
  int q = 0;       // streamed rows of this CTA
  for (int b = blockIdx.x; b < a.batch; b += gridDim.x) {
    if (!fused_streams(a, b)) {
      if (t == 0) {
        a.cand_gn[b] = -1;
        fused_fallback(a, b);
      }
      continue;
    }
    const tg_row_params p = a.params[b];
    const char* row;
    int head, nvec, tail0;
    row_geometry<DT>(a, b, row, head, nvec, tail0);
    const uint32_t* mask = nullptr;
    if (a.mask_table && a.state_id) {
      const int sid = a.state_id[b];
      if (sid >= 0) mask = a.mask_table + static_cast<int64_t>(sid) * a.mask_words;
    }
    const bool greedy = !(p.temperature > 0.0f);
    const bool topk = p.top_k > 0 && p.top_k < V;
    const int keff = greedy ? 1 : (topk ? p.top_k : V);
    const float tgt = kTgtMul * static_cast<float>(keff < V ? keff : kNoTopkTarget) + kTgtAdd;
    const int nsv = nvec < kFuChunkVecs ? nvec : kFuChunkVecs;
    const int sampled = nsv * EPV;

    // the slot of this row must have been released by the finisher of row q - NS
    const int s = q % NS;
    const long long w0 = clock64();
    if (t == 0) {
      bool ok = false;
      for (unsigned it = 0; it < kFuWaitLimit; it++) {
        if (ld_acquire_cta(&ctl.slot_free[s]) >= q / NS) { ok = true; break; }
        if (*reinterpret_cast<volatile int*>(&ctl.abort)) break;
        __nanosleep(128);
      }
      if (!ok && !ctl.abort) fail();
      fu_add(24, clock64() - w0);  // 24: filter waits for a free slot
      sm.cand_count = 0;
      sm.sn = *reinterpret_cast<volatile int*>(&ctl.abort);  // one reading for all filter threads
    }
    fbar();
    if (sm.sn) break;
    float* cand_y = reinterpret_cast<float*>(slots + static_cast<size_t>(s) * kCandMax * 8);
    int* cand_id = reinterpret_cast<int*>(cand_y + kCandMax);

    auto vmax_of = [&](const uint4& w, int j) {
      if (!mask) return E::vmax(w);
      float x[EPV];
      E::unpack(w, x);
      const uint32_t bits = mask_bits(mask, head + j * EPV, EPV);
      float vm = neg_inf();
#pragma unroll
      for (int e = 0; e < EPV; e++)
        if ((bits >> e) & 1u) vm = fmaxf(vm, x[e]);
      return vm;
    };
    auto append_vec = [&](const uint4& w, int j, float th) {
      float x[EPV];
      E::unpack(w, x);
      const uint32_t bits = mask ? mask_bits(mask, head + j * EPV, EPV) : 0xffu;
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
    auto drain = [&](int cnt, float th) {  // warp-uniform cnt <= kRing
      __syncwarp();
      for (int i0 = 0; i0 < cnt; i0 += 32) {
        const int i = i0 + lane;
        float x[EPV];
        uint32_t hits = 0;
        int j = 0;
        if (i < cnt) {
          j = ridx[i];
          E::unpack(rdata[i], x);
          const uint32_t bits = mask ? mask_bits(mask, head + j * EPV, EPV) : 0xffu;
#pragma unroll
          for (int e = 0; e < EPV; e++) hits |= (((bits >> e) & 1u) && x[e] >= th ? 1u : 0u) << e;
        }
        const int c = __popc(hits);
        int pre = 0, tot = 0;
#pragma unroll
        for (int bit = 0; bit < (EPV >= 8 ? 4 : 3); bit++) {
          const unsigned m = __ballot_sync(kFull, (c >> bit) & 1);
          pre += __popc(m & lt) << bit;
          tot += __popc(m) << bit;
        }
        int base = 0;
        if (lane == 0 && tot) base = atomicAdd(&sm.cand_count, tot);
        int pos = __shfl_sync(kFull, base, 0) + pre;
#pragma unroll
        for (int e = 0; e < EPV; e++) {
          if ((hits >> e) & 1u) {
            if (pos < kCandMax) { cand_y[pos] = x[e]; cand_id[pos] = head + j * EPV + e; }
            pos++;
          }
        }
      }
      __syncwarp();
    };

    float theta = neg_inf();
    int rcnt = 0;  // warp-uniform ring fill
    bool alive = true;
    for (int c = 0; c * kFuChunkVecs < nvec; c++, g++) {
      const int st = static_cast<int>(g % S);
      const long long f0 = clock64();
      const bool got = __all_sync(kFull, mbar_wait_parity(&ctl.full[st], (g / S) & 1u, &ctl.abort));
      const long long f1 = clock64();
      if (t == 0) fu_add(25, f1 - f0);  // 25: filter waits for a stage
      if (t == 224) fu_add(31, f1 - f0);  // 31: the same, seen by warp 7
      if (!got && t == 0 && !ctl.abort) fail();
      const uint4* cv = reinterpret_cast<const uint4*>(ring + static_cast<size_t>(st) * kFuChunkBytes);
      const int j0 = c * kFuChunkVecs;
      const int nv = min(kFuChunkVecs, nvec - j0);
      if (c == 0) {
        uint4 raw[kSampleVecs];
        float vm[kSampleVecs];
#pragma unroll
        for (int qv = 0; qv < kSampleVecs; qv++) {
          const int jl = t + qv * NT;
          if (jl < nv) raw[qv] = cv[jl];
          vm[qv] = jl < nv ? vmax_of(raw[qv], jl) : neg_inf();
        }
        if (V > kCandMax && sampled > 0) {
          int rr = static_cast<int>(ceilf(tgt * static_cast<float>(sampled) / static_cast<float>(V)));
          const unsigned rk = static_cast<unsigned>(rr < 1 ? 1 : rr);
          theta = sample_theta<kSampleVecs, NT, kFuBarFilter>(vm, rk, sm);
        }
#pragma unroll
        for (int qv = 0; qv < kSampleVecs; qv++) {
          const int jl = t + qv * NT;
          if (jl < nv && vm[qv] >= theta) append_vec(raw[qv], jl, theta);
        }
        // head and tail scalars
        int sc_id = -1;
        if (t < head) sc_id = t;
        else if (t - head < V - tail0) sc_id = tail0 + (t - head);
        if (sc_id >= 0) {
          float sc = E::load(row, sc_id);
          if (mask && !mask_allows(mask, sc_id)) sc = neg_inf();
          if (sc >= theta) {
            const int pos = atomicAdd(&sm.cand_count, 1);
            if (pos < kCandMax) { cand_y[pos] = sc; cand_id[pos] = sc_id; }
          }
        }
      } else {
        // one packed max and one ballot per vector; vectors holding an element
        // >= theta go raw (16 bytes + index) to the warp's ring, which the warp
        // expands 32 entries at a time (nearly every 4-vector group of a warp
        // holds a hit, so a per-warp skip test would not pay)
#pragma unroll
        for (int qv = 0; qv < kSampleVecs; qv++) {
          const int jl = t + qv * NT;
          uint4 w = kNegVec;
          if (jl < nv) w = cv[jl];
          const bool hit = vmax_of(w, j0 + jl) >= theta;
          const unsigned bal = __ballot_sync(kFull, hit);
          if (bal) {
            if (hit) {
              const int pos = rcnt + __popc(bal & lt);
              rdata[pos] = w;
              ridx[pos] = j0 + jl;
            }
            rcnt += __popc(bal);
            if (rcnt >= 32) { drain(rcnt, theta); rcnt = 0; }
          }
        }
      }
      if (t == 0) fu_add(c == 0 ? 29 : 30, clock64() - f1);  // 29: stage 0 (theta), 30: other stages
      // the stage goes back to the producer
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&ctl.empty[st])) : "memory");
      if (!got) { alive = false; g++; break; }
    }
    if (rcnt) drain(rcnt, theta);
    if (!alive) atomicOr(&ctl.abort, 1);
    fbar();  // the list is complete
    if (t == 0) sm.sn = *reinterpret_cast<volatile int*>(&ctl.abort);
    fbar();
    if (sm.sn) break;
    if (t == 0) fu_add(26, clock64() - w0);  // 26: filter time per row
    if (t == 0) {
      ctl.slot_row[s] = b;
      ctl.slot_n[s] = sm.cand_count;
      ctl.slot_theta[s] = theta;
      st_release_cta(&ctl.slot_pub[s], q + 1);
    }
    q++;
  }
  if (t == 0) {
    ctl.total = q;
    st_release_cta(&ctl.done, 1);
  }
}

}  // namespace tg
