// tg_theta.cuh -- the streaming kernel's per-row threshold, computed ahead of it.
//
// The top-k prefilter needs a threshold theta per row: a lower bound of the
// value of rank ~1.5k+96, estimated from a sample (the first 1024 128-bit
// vectors of the row, the maxima of their 8 or 4 elements).  Computed inside the
// streaming kernel it stalls that CTA's loads for its histogram and barriers
// (about an eighth of the CTA's time on config 4).  Here four warps per row read
// the sample (16 KB of bf16, 6 % of the row, left in L2 for the stream) and
// selects the rk-th largest vector maximum exactly (grp_select over 32-bit
// keys); the streaming kernel then starts on its loads at once.  With four
// warps per row each thread's 8 loads are in flight together.
//
// Any theta gives the same ids: the list holds every element >= theta, and a
// row whose list is short, overflows or could tie the k-th value below theta is
// retried or finished by the exact full-row path.  This theta is the rk-th
// largest sample maximum itself (sample_theta in tg_sample.cuh returns a lower
// bound of it, the smallest maximum of the histogram bin that holds it).
#pragma once

#include "tg_finish_warp.cuh"

namespace tg {

constexpr int kThetaG = 4;                     // warps per row
constexpr int kThetaRows = 2;                  // rows per CTA
constexpr int kThetaNT = kThetaRows * kThetaG * 32;
constexpr int kThetaVecsPerLane = kSampleVecs * kSampleNT / (32 * kThetaG);  // 8 of the 1024-vector sample

// kThetaG warps per row; writes a.cand_gth[b] (-inf when the sample holds fewer
// than rk finite maxima).
template <int DT>
__global__ void __launch_bounds__(kThetaNT) theta_kernel(SampleArgs a) {
  using E = Elt<DT>;
  constexpr int EPV = E::kEPV;
  __shared__ GrpSel wsel[kThetaRows];
  const int gi = threadIdx.x / (32 * kThetaG), gt = threadIdx.x % (32 * kThetaG);
  const int b = blockIdx.x * kThetaRows + gi;
  if (b >= a.batch) return;  // the whole group
  const Grp<kThetaG> g{gi, gt, gt >> 5, gt & 31, 1 + gi};
  const int lane = g.lane;
  const tg_row_params p = a.params[b];
  const int V = a.vocab;
  const char* row = reinterpret_cast<const char*>(a.logits) + b * a.row_stride * E::kSize;
  const uintptr_t addr = reinterpret_cast<uintptr_t>(row);
  int head = static_cast<int>(((16u - (addr & 15u)) & 15u) / E::kSize);
  if (head > V) head = V;
  const int nvec = (V - head) / EPV;
  const uint4* vrow = reinterpret_cast<const uint4*>(row + head * E::kSize);
  const uint32_t* mask = nullptr;
  if (a.mask_table && a.state_id) {
    const int sid = a.state_id[b];
    if (sid >= a.num_states) return;  // not streamed
    if (sid >= 0) mask = a.mask_table + static_cast<int64_t>(sid) * a.mask_words;
  }
  const bool greedy = !(p.temperature > 0.0f);
  const bool topk = p.top_k > 0 && p.top_k < V;
  const int keff = greedy ? 1 : (topk ? p.top_k : V);
  const float tgt = kTgtMul * static_cast<float>(keff < V ? keff : kNoTopkTargetStream) + kTgtAdd;  // feeds the stream
  const int nsv = nvec < kSampleVecs * kSampleNT ? nvec : kSampleVecs * kSampleNT;
  const int sampled = nsv * EPV;
  if (!(V > kCandMax && sampled > 0)) {
    if (gt == 0) a.cand_gth[b] = neg_inf();
    return;
  }
  int rr = static_cast<int>(ceilf(tgt * static_cast<float>(sampled) / static_cast<float>(V)));
  const unsigned rk = static_cast<unsigned>(rr < 1 ? 1 : rr);

  // the sample's vector maxima: each thread's 8 loads in flight together
  float vm[kThetaVecsPerLane];
  {
    uint4 w[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const int j = gt + 32 * kThetaG * q;
      if (j < nsv) w[q] = __ldg(vrow + j);
    }
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const int j = gt + 32 * kThetaG * q;
      float m = neg_inf();
      if (j < nsv) {
        if (!mask) {
          m = E::vmax(w[q]);
        } else {
          float x[EPV];
          E::unpack(w[q], x);
          const uint32_t bits = mask_bits(mask, head + j * EPV, EPV);
#pragma unroll
          for (int e = 0; e < EPV; e++)
            if ((bits >> e) & 1u) m = fmaxf(m, x[e]);
        }
      }
      vm[q] = m;
    }
  }
  float mx = neg_inf(), nmn = neg_inf();
  unsigned int fin = 0;
#pragma unroll
  for (int q = 0; q < kThetaVecsPerLane; q++) {
    if (vm[q] > neg_inf()) {
      mx = fmaxf(mx, vm[q]);
      nmn = fmaxf(nmn, -vm[q]);
      fin++;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(kFull, mx, o));
    nmn = fmaxf(nmn, __shfl_xor_sync(kFull, nmn, o));
    fin += __shfl_xor_sync(kFull, fin, o);
  }
  GrpSel& ws = wsel[gi];
  if (lane == 0) { ws.rf[g.gw] = mx; ws.rg[g.gw] = nmn; ws.ri[g.gw] = static_cast<int>(fin); }
  g.sync();
  mx = neg_inf();
  nmn = neg_inf();
  fin = 0;
#pragma unroll
  for (int w = 0; w < kThetaG; w++) {
    mx = fmaxf(mx, ws.rf[w]);
    nmn = fmaxf(nmn, ws.rg[w]);
    fin += static_cast<unsigned>(ws.ri[w]);
  }
  g.sync();
  float theta = neg_inf();
  if (fin >= rk) {
    uint32_t key;
    unsigned long long before, w;
    const bool ok = grp_select<false, uint32_t>(
        g,
        [&](auto&& f) {
#pragma unroll
          for (int q = 0; q < kThetaVecsPerLane; q++)
            if (vm[q] > neg_inf()) f(~fkey(vm[q]), vm[q]);
        },
        [](uint32_t, float) { return 1ull; }, ~fkey(mx), ~fkey(-nmn), false,
        [&](unsigned long long c) { return c >= rk; }, ws, key, before, w);
    if (ok) theta = key2f(~key);
  }
  if (gt == 0) a.cand_gth[b] = theta;
}

}  // namespace tg
