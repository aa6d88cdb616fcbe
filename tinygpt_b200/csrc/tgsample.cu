// tgsample.cu -- C ABI of the sampling engine (include/tgsample.h).
//
// Host side: argument checks, launch configuration and the host-buffer
// variants.  No allocation happens in tg_sample / tg_spec_verify except the
// first growth of the verification statistics buffer.
#include <cuda_runtime.h>

#include <dlfcn.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <chrono>
#include <thread>

#include "../../include/tgsample.h"
#include "tg_sample.cuh"
#include "tg_finish_warp.cuh"
#include "tg_fused.cuh"
#include "tg_theta.cuh"
#include "tg_spec.cuh"

namespace {

thread_local std::string g_last_error;

int32_t fail(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int32_t cuda_fail(cudaError_t e, const char* what) {
  return fail(TG_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define TG_CUDA(call)                                 \
  do {                                                \
    cudaError_t e_ = (call);                          \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

class DeviceGuard {
 public:
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev_);
    if (prev_ != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != prev_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0;
};

// Device buffer that only grows.
struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
  cudaError_t ensure(size_t n) {
    if (n <= cap) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
    cudaError_t e = cudaMalloc(&p, n);
    if (e == cudaSuccess) cap = n;
    return e;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    cap = 0;
  }
};

// Scratch of tg_spec_verify_static: TG_STATIC_SPEC_MAX_ROWS statistics records
// followed by one status word.  In host code this name is only a stand-in for
// the device array; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_static_spec_scratch[
    TG_STATIC_SPEC_MAX_ROWS * sizeof(tg::SpecStat) + 256];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kMaxDevices] = {};

// Device address of the static scratch on the current device `dev` (looked up
// once per device, with that device current).
cudaError_t static_scratch(int dev, void** out) {
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_spec_scratch);
    if (e != cudaSuccess) return e;
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return cudaSuccess;
}

}  // namespace

struct tg_sampler {
  int device = 0;
  int vocab = 0;
  int max_batch = 0;
  uint32_t* d_status = nullptr;  // device error word
  unsigned long long* d_counters = nullptr;  // TG_PATH_* counters
  DevBuf stats;                  // spec-verify statistics (+ per-row state of the lazy mode)
  // staging for tg_sample_host
  DevBuf h_logits, h_params, h_hist, h_hlen, h_mask, h_state, h_unif, h_out, h_prob;
  cudaStream_t stream = nullptr;  // used by tg_sample_host only
  // two-kernel mode: raw candidate lists of up to split_rows rows per launch pair
  DevBuf cand;
  DevBuf shard_recs;   // tg_sample_sharded: local records, then the gathered ones
  int split_rows = 0;  // 0: single-kernel mode
  // tg_sampler_profile: events around the kernels of the last tg_sample call
  bool profile = false;
  cudaEvent_t prof_ev[3] = {nullptr, nullptr, nullptr};
  int prof_kind = 0;  // 0: no call recorded, 1: one kernel, 2: two kernels
  int coll_timeout_ms = 0;        // tg_sample_sharded: 0 = no host wait
  cudaEvent_t coll_ev = nullptr;
  std::mutex mu;
};

namespace {
// An environment switch set to "0" turns the feature off (diagnostics).
bool getenv_off(const char* name) {
  const char* v = getenv(name);
  return v && v[0] == '0';
}

// Launches `kernel` on `st` as a programmatic dependent of the previous work on
// the stream: its launch is processed while that work drains, and the kernel
// waits on the device (griddepcontrol.wait) before it reads anything.
template <class... KArgs, class... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), int grid, int block, size_t smem, cudaStream_t st,
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

// Rows per streaming / finishing launch pair (bounds the candidate buffer:
// kCandMax * 8 + 8 bytes per row).
constexpr int kSplitRows = 2048;
// The two-kernel mode pays for itself from this many rows on.
constexpr int kSplitMinBatchDefault = 1024;
// TG_SPLIT_MIN_BATCH overrides it (diagnostics: the two-kernel mode on small batches).
int split_min_batch() {
  static const int v = [] {
    const char* e = getenv("TG_SPLIT_MIN_BATCH");
    return e ? atoi(e) : kSplitMinBatchDefault;
  }();
  return v;
}
}  // namespace

extern "C" {

int32_t tg_abi_version(void) { return (1 << 16) | 0; }

const char* tg_last_error_string(void) { return g_last_error.c_str(); }

int32_t tg_sampler_create(int32_t device, int32_t vocab, int32_t max_batch, tg_sampler** out) {
  if (!out) return fail(TG_ERR_INVALID_ARG, "out is NULL");
  *out = nullptr;
  if (vocab <= 0 || vocab > TG_MAX_VOCAB) return fail(TG_ERR_UNSUPPORTED, "vocab outside [1, TG_MAX_VOCAB]");
  if (max_batch <= 0) return fail(TG_ERR_INVALID_ARG, "max_batch must be positive");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fail(TG_ERR_NO_DEVICE, "CUDA device not present");
  DeviceGuard g(device);
  tg_sampler* s = new tg_sampler();
  s->device = device;
  s->vocab = vocab;
  s->max_batch = max_batch;
  cudaError_t e = cudaMalloc(&s->d_status, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(s->d_status, 0, sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMalloc(&s->d_counters, sizeof(unsigned long long) * TG_PATH_COUNTERS);
  if (e == cudaSuccess) e = cudaMemset(s->d_counters, 0, sizeof(unsigned long long) * TG_PATH_COUNTERS);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
  const int max_smem = 200 * 1024;
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tg::sample_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tg::sample_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tg::sample_list_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tg::sample_list_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tg::sample_kernel<0, false, tg::kWideNT>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(tg::sample_kernel<1, false, tg::kWideNT>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  // the two-kernel mode serves rows longer than a candidate list, in batches of
  // split_min_batch() rows or more (TG_SAMPLE_SPLIT=0 turns it off)
  const char* split_env = getenv("TG_SAMPLE_SPLIT");
  if (e == cudaSuccess && vocab > tg::kCandMax && max_batch >= split_min_batch() &&
      !(split_env && split_env[0] == '0')) {
    s->split_rows = max_batch < kSplitRows ? max_batch : kSplitRows;
    // per row: the list (value, id), its length and theta, a fallback-list slot; one count
    e = s->cand.ensure(static_cast<size_t>(s->split_rows) * (static_cast<size_t>(tg::kCandMax) * 8 + 12) + 16);
  }
  if (e == cudaSuccess && s->split_rows) {
    e = cudaFuncSetAttribute(tg::finish_warp_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, tg::kWfSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tg::finish_warp_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, tg::kWfSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tg::finish_warp_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, tg::kWfSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tg::finish_warp_kernel<3>, cudaFuncAttributeMaxDynamicSharedMemorySize, tg::kWfSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tg::sample_fused_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, tg::kFuSmem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tg::sample_fused_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, tg::kFuSmem);
  }
  if (e != cudaSuccess) {
    tg_sampler_destroy(s);
    return cuda_fail(e, "tg_sampler_create");
  }
  *out = s;
  return TG_OK;
}

int32_t tg_sampler_destroy(tg_sampler* s) {
  if (!s) return TG_OK;
  {
    DeviceGuard g(s->device);
    if (s->d_status) cudaFree(s->d_status);
    if (s->d_counters) cudaFree(s->d_counters);
    s->stats.release();
    s->cand.release();
    s->shard_recs.release();
    for (cudaEvent_t ev : s->prof_ev)
      if (ev) cudaEventDestroy(ev);
    if (s->coll_ev) cudaEventDestroy(s->coll_ev);
    for (DevBuf* b : {&s->h_logits, &s->h_params, &s->h_hist, &s->h_hlen, &s->h_mask, &s->h_state,
                      &s->h_unif, &s->h_out, &s->h_prob})
      b->release();
    if (s->stream) cudaStreamDestroy(s->stream);
  }
  delete s;
  return TG_OK;
}

static int32_t launch_sample(tg_sampler* s, int32_t vocab_offset, int32_t full_vocab,
                             tg_shard_record* shard_out, const void* logits, int32_t dtype, int64_t row_stride,
                  int32_t batch, const tg_row_params* params, const int32_t* history,
                  const int32_t* history_len, int32_t history_stride,
                  const uint32_t* mask_table, int32_t num_states, const int32_t* state_id,
                  const float* uniforms, int32_t* out_ids, float* out_probs, void* stream) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  if (dtype != TG_DTYPE_F32 && dtype != TG_DTYPE_BF16) return fail(TG_ERR_INVALID_ARG, "dtype must be TG_DTYPE_F32 or TG_DTYPE_BF16");
  if (batch < 0 || batch > s->max_batch) return fail(TG_ERR_INVALID_ARG, "batch outside [0, max_batch]");
  if (batch == 0) return TG_OK;
  if (!logits || !params || (!out_ids && !shard_out)) return fail(TG_ERR_INVALID_ARG, "logits, params and out_ids are required");
  if (row_stride < s->vocab) return fail(TG_ERR_INVALID_ARG, "row_stride < vocab");
  const bool has_hist = history_len != nullptr;
  if (has_hist && (!history || history_stride <= 0)) return fail(TG_ERR_INVALID_ARG, "history_len given without history / history_stride");
  const bool has_mask = state_id != nullptr;
  if (has_mask && (!mask_table || num_states <= 0)) return fail(TG_ERR_INVALID_ARG, "state_id given without mask_table / num_states");

  tg::SampleArgs a{};
  a.logits = logits;
  a.row_stride = row_stride;
  a.vocab = s->vocab;
  a.batch = batch;
  a.params = params;
  a.history = has_hist ? history : nullptr;
  a.history_len = has_hist ? history_len : nullptr;
  a.history_stride = has_hist ? history_stride : 0;
  a.hist_cap = has_hist ? (history_stride < TG_MAX_HISTORY ? history_stride : TG_MAX_HISTORY) : 0;
  a.ht_log2 = 0;
  if (a.hist_cap > 0) {
    int l = 5;
    while ((1 << l) < 2 * a.hist_cap) l++;
    a.ht_log2 = l;
  }
  a.mask_table = has_mask ? mask_table : nullptr;
  a.num_states = has_mask ? num_states : 0;
  a.mask_words = (full_vocab + 31) / 32;
  a.vocab_offset = vocab_offset;
  a.full_vocab = full_vocab;
  a.shard_out = shard_out;
  a.state_id = has_mask ? state_id : nullptr;
  a.uniforms = uniforms;
  a.out_ids = out_ids;
  a.out_probs = out_probs;
  a.status = s->d_status;
  {
    const char* ds = getenv("TG_WF_STOP");
    a.debug_stop = ds ? atoi(ds) : 0;
  }
  a.counters = s->d_counters;
  const size_t smem = static_cast<size_t>(tg::kCandMax) * 12 + (a.ht_log2 ? (size_t(8) << a.ht_log2) : 0);
  DeviceGuard g(s->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (s->profile) TG_CUDA(cudaEventRecord(s->prof_ev[0], st));
  if (batch >= tg::kWideMinBatch && batch <= tg::kWideMaxBatch && s->vocab > tg::kCandMax) {
    // few rows: one 1024-thread CTA per row, four times the warps on each row's
    // latency-bound stages (the rest-of-row mass of rows without top-k above all);
    // the warp rings follow the hash in shared memory
    const size_t wsmem = smem + static_cast<size_t>(tg::kWideNT / 32) * tg::kRing * 20;
    if (dtype == TG_DTYPE_F32)
      tg::sample_kernel<0, false, tg::kWideNT><<<batch, tg::kWideNT, wsmem, st>>>(a);
    else
      tg::sample_kernel<1, false, tg::kWideNT><<<batch, tg::kWideNT, wsmem, st>>>(a);
    TG_CUDA(cudaGetLastError());
    if (s->profile) {
      TG_CUDA(cudaEventRecord(s->prof_ev[1], st));
      s->prof_kind = 1;
    }
    return TG_OK;
  }
  if (s->split_rows == 0 || batch < split_min_batch()) {
    if (dtype == TG_DTYPE_F32)
      tg::sample_kernel<0><<<batch, tg::kSampleNT, smem, st>>>(a);
    else
      tg::sample_kernel<1><<<batch, tg::kSampleNT, smem, st>>>(a);
    TG_CUDA(cudaGetLastError());
    if (s->profile) {
      TG_CUDA(cudaEventRecord(s->prof_ev[1], st));
      s->prof_kind = 1;
    }
    return TG_OK;
  }
  // two-kernel mode, split_rows rows per launch pair: the streaming kernel
  // (rings in shared memory, high occupancy) leaves the raw candidates of each
  // row in s->cand; the finishing kernel then selects from them.  Running the
  // pair back to back beat running chunks of the two concurrently, which
  // split the SMs between them.
  const int R = s->split_rows;
  char* cb = static_cast<char*>(s->cand.p);
  a.cand_gy = reinterpret_cast<float*>(cb);
  a.cand_gid = reinterpret_cast<int32_t*>(cb + static_cast<size_t>(R) * tg::kCandMax * 4);
  a.cand_gn = reinterpret_cast<int32_t*>(cb + static_cast<size_t>(R) * tg::kCandMax * 8);
  a.cand_gth = reinterpret_cast<float*>(cb + static_cast<size_t>(R) * (tg::kCandMax * 8 + 4));
  // the warp finisher takes the rows of a call whose history hash fits a warp's
  // share of shared memory; the vocab-sharded mode keeps the CTA finisher
  const bool warp_fin = !shard_out && a.ht_log2 <= 11 && !getenv_off("TG_WARP_FINISH");
  if (warp_fin) {
    a.fb_rows = reinterpret_cast<int32_t*>(cb + static_cast<size_t>(R) * (tg::kCandMax * 8 + 8));
    a.fb_count = reinterpret_cast<int32_t*>(cb + static_cast<size_t>(R) * (tg::kCandMax * 8 + 12));
  }
  int nsm = 148;
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, s->device);
  // the fused kernel (streaming and finishing in one persistent launch): the
  // most ring stages (3..6) that fit next to 4 list slots and 3 finisher groups
  tg::FusedCfg fcfg{};
  // (opt-in with TG_FUSED=1: measured slower than the two launches so far --
  // 458 vs 194 us per config-4 call -- its filter and finisher warps are too
  // few per SM to hide their latency)
  const char* fenv = getenv("TG_FUSED");
  bool fused = warp_fin && fenv && fenv[0] == '1';
  if (fused) {
    int st = 6;
    while (st >= 3 && tg::fused_smem(st, 4, 3, a.ht_log2, nullptr) > static_cast<size_t>(tg::kFuSmem)) st--;
    fused = st >= 3;
    if (fused) tg::fused_smem(st, 4, 3, a.ht_log2, &fcfg);
    const char* dbg = getenv("TG_FUSED_DEBUG");
    fcfg.debug = dbg ? atoi(dbg) : 0;
  }
  const size_t fsmem = fused ? tg::fused_smem(fcfg.stages, fcfg.slots, fcfg.groups, a.ht_log2, nullptr) : 0;
  const size_t ring_smem = static_cast<size_t>(tg::kSampleNT / 32) * tg::kStreamRing * 20;
  // the threshold kernel ahead of the stream: opt-in (TG_THETA_FIRST=1).  It
  // shortens the stream by 13 us on config 4 but costs 17-20 us itself.
  const char* thenv = getenv("TG_THETA_FIRST");
  const bool theta_first = thenv && thenv[0] == '1';
  const int64_t es = dtype == TG_DTYPE_F32 ? 4 : 2;
  for (int32_t r0 = 0; r0 < batch; r0 += R) {
    const int32_t n = batch - r0 < R ? batch - r0 : R;
    tg::SampleArgs c = a;
    c.batch = n;
    c.logits = static_cast<const char*>(logits) + r0 * row_stride * es;
    c.params = params + r0;
    if (c.history) c.history = history + static_cast<int64_t>(r0) * history_stride;
    if (c.history_len) c.history_len = history_len + r0;
    if (c.state_id) c.state_id = state_id + r0;
    if (c.uniforms) c.uniforms = uniforms + r0;
    if (c.out_ids) c.out_ids = out_ids + r0;
    if (c.out_probs) c.out_probs = out_probs + r0;
    if (c.shard_out) c.shard_out = shard_out + r0;
    const bool mark = s->profile && r0 == 0 && n == batch;  // single launch pair: time each kernel
    if (fused) {  // one persistent kernel per SM, then the rows it left on CTAs
      TG_CUDA(cudaMemsetAsync(c.fb_count, 0, sizeof(int32_t), st));
      const int grid = n < nsm ? n : nsm;
      const int threads = tg::kFuFinTid0 + fcfg.groups * 32 * tg::kFuG;
      if (dtype == TG_DTYPE_F32)
        tg::sample_fused_kernel<0><<<grid, threads, fsmem, st>>>(c, fcfg);
      else
        tg::sample_fused_kernel<1><<<grid, threads, fsmem, st>>>(c, fcfg);
      if (mark) TG_CUDA(cudaEventRecord(s->prof_ev[1], st));
      const int g = n;  // one CTA per possible fallback row
      if (dtype == TG_DTYPE_F32)
        tg::sample_list_kernel<0><<<g, tg::kSampleNT, smem, st>>>(c);
      else
        tg::sample_list_kernel<1><<<g, tg::kSampleNT, smem, st>>>(c);
      TG_CUDA(cudaGetLastError());
      continue;
    }
    if (theta_first) {  // every row's threshold first (one warp per row), then the pure stream
      c.theta_given = 1;
      const int tg_grid = (n + tg::kThetaRows - 1) / tg::kThetaRows;
      if (dtype == TG_DTYPE_F32)
        tg::theta_kernel<0><<<tg_grid, tg::kThetaNT, 0, st>>>(c);
      else
        tg::theta_kernel<1><<<tg_grid, tg::kThetaNT, 0, st>>>(c);
    }
    TG_CUDA(dtype == TG_DTYPE_F32
                ? launch_dependent(tg::sample_kernel<0, true>, n, tg::kSampleNT, ring_smem, st, c)
                : launch_dependent(tg::sample_kernel<1, true>, n, tg::kSampleNT, ring_smem, st, c));
    if (mark) TG_CUDA(cudaEventRecord(s->prof_ev[1], st));
    if (warp_fin) {  // a warp per row, then the rows it left on CTAs
      // one CTA per SM with ceil(n / SMs) rows; G warps per row, G the largest
      // of 4, 2, 1 that keeps the CTA within 28 warps (register file at the
      // kernel's register count) and 16 warps per row group in all
      int rpc = (n + nsm - 1) / nsm;
      rpc = rpc < 1 ? 1 : (rpc > tg::kWfMaxWarps ? tg::kWfMaxWarps : rpc);
      const int G = rpc * 4 <= tg::kWfGroupWarps ? 4 : rpc * 3 <= tg::kWfGroupWarps ? 3 : (rpc * 2 <= tg::kWfGroupWarps ? 2 : 1);
      const size_t wsb = static_cast<size_t>(rpc) * tg::grp_fin_bytes(a.ht_log2);
      const int pool = static_cast<int>((static_cast<size_t>(tg::kWfSmem) - wsb) / 8);
      const int grid = (n + rpc - 1) / rpc;
      cudaError_t le;
      if (G == 4)
        le = launch_dependent(tg::finish_warp_kernel<4>, grid, rpc * 128, tg::kWfSmem, st, c, pool);
      else if (G == 3)
        le = launch_dependent(tg::finish_warp_kernel<3>, grid, rpc * 96, tg::kWfSmem, st, c, pool);
      else if (G == 2)
        le = launch_dependent(tg::finish_warp_kernel<2>, grid, rpc * 64, tg::kWfSmem, st, c, pool);
      else
        le = launch_dependent(tg::finish_warp_kernel<1>, grid, rpc * 32, tg::kWfSmem, st, c, pool);
      TG_CUDA(le);
      const int g = n;  // one CTA per possible fallback row
      if (dtype == TG_DTYPE_F32)
        le = launch_dependent(tg::sample_list_kernel<0>, g, tg::kSampleNT, smem, st, c);
      else
        le = launch_dependent(tg::sample_list_kernel<1>, g, tg::kSampleNT, smem, st, c);
      TG_CUDA(le);
    } else if (dtype == TG_DTYPE_F32) {
      tg::sample_kernel<0><<<n, tg::kSampleNT, smem, st>>>(c);
    } else {
      tg::sample_kernel<1><<<n, tg::kSampleNT, smem, st>>>(c);
    }
    TG_CUDA(cudaGetLastError());
  }
  if (s->profile) {
    if (batch <= R) {
      TG_CUDA(cudaEventRecord(s->prof_ev[2], st));
      s->prof_kind = 2;
    } else {  // several launch pairs: the whole call only
      TG_CUDA(cudaEventRecord(s->prof_ev[1], st));
      s->prof_kind = 1;
    }
  }
  return TG_OK;
}

int32_t tg_sample(tg_sampler* s, const void* logits, int32_t dtype, int64_t row_stride,
                  int32_t batch, const tg_row_params* params, const int32_t* history,
                  const int32_t* history_len, int32_t history_stride,
                  const uint32_t* mask_table, int32_t num_states, const int32_t* state_id,
                  const float* uniforms, int32_t* out_ids, float* out_probs, void* stream) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  return launch_sample(s, 0, s->vocab, nullptr, logits, dtype, row_stride, batch, params, history,
                       history_len, history_stride, mask_table, num_states, state_id, uniforms,
                       out_ids, out_probs, stream);
}

int32_t tg_sample_shard_local(tg_sampler* s, int32_t vocab_offset, int32_t full_vocab,
                              const void* logits, int32_t dtype, int64_t row_stride,
                              int32_t batch, const tg_row_params* params,
                              const int32_t* history, const int32_t* history_len,
                              int32_t history_stride, const uint32_t* mask_table,
                              int32_t num_states, const int32_t* state_id,
                              tg_shard_record* out_records, void* stream) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  if (!out_records) return fail(TG_ERR_INVALID_ARG, "out_records is NULL");
  if (vocab_offset < 0 || full_vocab > TG_MAX_VOCAB || static_cast<int64_t>(vocab_offset) + s->vocab > full_vocab)
    return fail(TG_ERR_INVALID_ARG, "shard [vocab_offset, vocab_offset + vocab) outside [0, full_vocab <= TG_MAX_VOCAB)");
  return launch_sample(s, vocab_offset, full_vocab, out_records, logits, dtype, row_stride, batch,
                       params, history, history_len, history_stride, mask_table, num_states,
                       state_id, nullptr, nullptr, nullptr, stream);
}

int32_t tg_sample_shard_merge(tg_sampler* s, const tg_shard_record* records, int32_t nshards,
                              int32_t full_vocab, int32_t batch, const tg_row_params* params,
                              const float* uniforms, int32_t* out_ids, float* out_probs,
                              void* stream) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  if (batch < 0 || batch > s->max_batch) return fail(TG_ERR_INVALID_ARG, "batch outside [0, max_batch]");
  if (nshards <= 0 || full_vocab <= 0 || full_vocab > TG_MAX_VOCAB) return fail(TG_ERR_INVALID_ARG, "bad nshards / full_vocab");
  if (batch == 0) return TG_OK;
  if (!records || !params || !out_ids) return fail(TG_ERR_INVALID_ARG, "records, params and out_ids are required");
  DeviceGuard g(s->device);
  tg::MergeArgs m{records, nshards, batch, full_vocab, params, uniforms, out_ids, out_probs, s->d_status};
  tg::sample_merge_kernel<<<batch, tg::kSampleNT, static_cast<size_t>(tg::kCandMax) * 12,
                            static_cast<cudaStream_t>(stream)>>>(m);
  TG_CUDA(cudaGetLastError());
  return TG_OK;
}

// ncclAllGather of the NCCL the host process has loaded (the one that made the
// caller's communicator), found at run time so this library links no NCCL.
// NCCL's ABI: ncclResult_t (0 = success), ncclUint8 = 1.
typedef int (*tg_nccl_allgather_fn)(const void*, void*, size_t, int, void*, cudaStream_t);

// Global symbols first, then an NCCL already loaded with local scope (found by
// its soname; RTLD_NOLOAD never loads a new copy).  A miss is not cached.
static tg_nccl_allgather_fn nccl_allgather() {
  static tg_nccl_allgather_fn fn = nullptr;
  if (fn) return fn;
  void* sym = dlsym(RTLD_DEFAULT, "ncclAllGather");
  for (const char* name : {"libnccl.so.2", "libnccl.so"}) {
    if (sym) break;
    void* h = dlopen(name, RTLD_LAZY | RTLD_NOLOAD);
    if (h) sym = dlsym(h, "ncclAllGather");
  }
  fn = reinterpret_cast<tg_nccl_allgather_fn>(sym);
  return fn;
}

typedef int (*tg_nccl_count_fn)(void*, int*);
typedef int (*tg_nccl_abort_fn)(void*);

// A symbol of the NCCL the process has loaded (global scope first, then an
// NCCL loaded with local scope, found by its soname), or nullptr.
static void* nccl_symbol(const char* name) {
  void* sym = dlsym(RTLD_DEFAULT, name);
  for (const char* lib : {"libnccl.so.2", "libnccl.so"}) {
    if (sym) break;
    void* h = dlopen(lib, RTLD_LAZY | RTLD_NOLOAD);
    if (h) sym = dlsym(h, name);
  }
  return sym;
}
static tg_nccl_count_fn nccl_comm_count() { return reinterpret_cast<tg_nccl_count_fn>(nccl_symbol("ncclCommCount")); }
static tg_nccl_abort_fn nccl_comm_abort() { return reinterpret_cast<tg_nccl_abort_fn>(nccl_symbol("ncclCommAbort")); }

// Waits for the work queued on `stream` (the all-gather) for at most the
// handle's collective timeout.  On expiry the communicator is aborted (its
// pending collectives then end with an error) and TG_ERR_COLLECTIVE returned.
static int32_t wait_collective(tg_sampler* s, void* comm, cudaStream_t stream) {
  DeviceGuard g(s->device);
  if (!s->coll_ev) TG_CUDA(cudaEventCreateWithFlags(&s->coll_ev, cudaEventDisableTiming));
  TG_CUDA(cudaEventRecord(s->coll_ev, stream));
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t q = cudaEventQuery(s->coll_ev);
    if (q == cudaSuccess) return TG_OK;
    if (q != cudaErrorNotReady) return cuda_fail(q, "cudaEventQuery (collective)");
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms >= s->coll_timeout_ms) break;
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  const tg_nccl_abort_fn abort_fn = nccl_comm_abort();
  if (abort_fn) abort_fn(comm);
  return fail(TG_ERR_COLLECTIVE, "the all-gather did not complete within the collective timeout; the communicator was aborted");
}

int32_t tg_sample_sharded(tg_sampler* s, void* nccl_comm, int32_t nranks, int32_t vocab_offset,
                          int32_t full_vocab, const void* logits, int32_t dtype, int64_t row_stride,
                          int32_t batch, const tg_row_params* params, const int32_t* history,
                          const int32_t* history_len, int32_t history_stride,
                          const uint32_t* mask_table, int32_t num_states, const int32_t* state_id,
                          const float* uniforms, int32_t* out_ids, float* out_probs, void* stream) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  if (!nccl_comm || nranks <= 0) return fail(TG_ERR_INVALID_ARG, "nccl_comm and nranks > 0 are required");
  if (batch < 0 || batch > s->max_batch) return fail(TG_ERR_INVALID_ARG, "batch outside [0, max_batch]");
  if (vocab_offset < 0 || full_vocab > TG_MAX_VOCAB || static_cast<int64_t>(vocab_offset) + s->vocab > full_vocab)
    return fail(TG_ERR_INVALID_ARG, "shard [vocab_offset, vocab_offset + vocab) outside [0, full_vocab <= TG_MAX_VOCAB)");
  if (batch == 0) return TG_OK;
  if (!out_ids) return fail(TG_ERR_INVALID_ARG, "out_ids is required");
  const tg_nccl_allgather_fn allgather = nccl_allgather();
  if (!allgather) return fail(TG_ERR_UNSUPPORTED, "no NCCL library is loaded in this process (ncclAllGather not found)");
  // the all-gather writes one record block per rank of the communicator
  const tg_nccl_count_fn count = nccl_comm_count();
  if (count) {
    int n = 0;
    const int cr = count(nccl_comm, &n);
    if (cr != 0) return fail(TG_ERR_CUDA, "ncclCommCount failed (ncclResult_t " + std::to_string(cr) + ")");
    if (n != nranks) return fail(TG_ERR_INVALID_ARG, "nranks differs from the communicator's size");
  }
  const size_t rec = sizeof(tg_shard_record) * static_cast<size_t>(batch);
  // one lock from the buffer check to the merge launch: the record buffer is
  // the handle's, shared by every call on it
  std::lock_guard<std::mutex> lk(s->mu);
  if (rec * (1 + static_cast<size_t>(nranks)) > s->shard_recs.cap)
    return fail(TG_ERR_UNSUPPORTED, "shard records not reserved for this batch and nranks (call tg_sampler_reserve)");
  tg_shard_record* local = static_cast<tg_shard_record*>(s->shard_recs.p);
  tg_shard_record* all = local + batch;
  int32_t rc = launch_sample(s, vocab_offset, full_vocab, local, logits, dtype, row_stride, batch, params,
                             history, history_len, history_stride, mask_table, num_states, state_id,
                             nullptr, nullptr, nullptr, stream);
  if (rc != TG_OK) return rc;
  DeviceGuard g(s->device);
  const int nr = allgather(local, all, rec, 1 /* ncclUint8 */, nccl_comm, static_cast<cudaStream_t>(stream));
  if (nr != 0) return fail(TG_ERR_CUDA, "ncclAllGather failed (ncclResult_t " + std::to_string(nr) + ")");
  if (s->coll_timeout_ms > 0) {  // bounded wait for the collective; on expiry the communicator is aborted
    rc = wait_collective(s, nccl_comm, static_cast<cudaStream_t>(stream));
    if (rc != TG_OK) return rc;
  }
  return tg_sample_shard_merge(s, all, nranks, full_vocab, batch, params, uniforms, out_ids, out_probs, stream);
}

int32_t tg_sampler_reserve(tg_sampler* s, int32_t max_K, int32_t max_ranks) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  if (max_K < 0 || max_K > 64 || max_ranks < 0) return fail(TG_ERR_INVALID_ARG, "max_K outside [0, 64] or max_ranks < 0");
  std::lock_guard<std::mutex> lk(s->mu);
  DeviceGuard g(s->device);
  const size_t B = static_cast<size_t>(s->max_batch);
  TG_CUDA(s->stats.ensure(sizeof(tg::SpecStat) * B * (2 * static_cast<size_t>(max_K) + 1) + sizeof(int32_t) * 2 * B));
  if (max_ranks > 0) TG_CUDA(s->shard_recs.ensure(sizeof(tg_shard_record) * B * (1 + static_cast<size_t>(max_ranks))));
  return TG_OK;
}

int32_t tg_sampler_set_collective_timeout(tg_sampler* s, int32_t timeout_ms) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  if (timeout_ms < 0) return fail(TG_ERR_INVALID_ARG, "timeout_ms < 0");
  s->coll_timeout_ms = timeout_ms;
  return TG_OK;
}

int32_t tg_sample_host(tg_sampler* s, const void* logits, int32_t dtype, int64_t row_stride,
                       int32_t batch, const tg_row_params* params, const int32_t* history,
                       const int32_t* history_len, int32_t history_stride,
                       const uint32_t* mask_table, int32_t num_states, const int32_t* state_id,
                       const float* uniforms, int32_t* out_ids, float* out_probs) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  if (batch <= 0) return batch == 0 ? TG_OK : fail(TG_ERR_INVALID_ARG, "batch < 0");
  if (!logits || !params || !out_ids) return fail(TG_ERR_INVALID_ARG, "logits, params and out_ids are required");
  if (dtype != TG_DTYPE_F32 && dtype != TG_DTYPE_BF16) return fail(TG_ERR_INVALID_ARG, "bad dtype");
  if (batch > s->max_batch) return fail(TG_ERR_INVALID_ARG, "batch > max_batch");
  if (row_stride < s->vocab) return fail(TG_ERR_INVALID_ARG, "row_stride < vocab");
  std::lock_guard<std::mutex> lk(s->mu);
  DeviceGuard g(s->device);
  cudaStream_t st = s->stream;
  const size_t esz = dtype == TG_DTYPE_F32 ? 4 : 2;
  const size_t nlog = static_cast<size_t>(batch) * row_stride * esz;
  TG_CUDA(s->h_logits.ensure(nlog));
  TG_CUDA(s->h_params.ensure(sizeof(tg_row_params) * batch));
  TG_CUDA(s->h_out.ensure(sizeof(int32_t) * batch));
  TG_CUDA(cudaMemcpyAsync(s->h_logits.p, logits, nlog, cudaMemcpyHostToDevice, st));
  TG_CUDA(cudaMemcpyAsync(s->h_params.p, params, sizeof(tg_row_params) * batch, cudaMemcpyHostToDevice, st));
  const int32_t* d_hist = nullptr;
  const int32_t* d_hlen = nullptr;
  if (history_len) {
    if (!history || history_stride <= 0) return fail(TG_ERR_INVALID_ARG, "history_len given without history");
    const size_t nh = sizeof(int32_t) * static_cast<size_t>(batch) * history_stride;
    TG_CUDA(s->h_hist.ensure(nh));
    TG_CUDA(s->h_hlen.ensure(sizeof(int32_t) * batch));
    TG_CUDA(cudaMemcpyAsync(s->h_hist.p, history, nh, cudaMemcpyHostToDevice, st));
    TG_CUDA(cudaMemcpyAsync(s->h_hlen.p, history_len, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    d_hist = static_cast<const int32_t*>(s->h_hist.p);
    d_hlen = static_cast<const int32_t*>(s->h_hlen.p);
  }
  const uint32_t* d_mask = nullptr;
  const int32_t* d_state = nullptr;
  if (state_id) {
    if (!mask_table || num_states <= 0) return fail(TG_ERR_INVALID_ARG, "state_id given without mask_table");
    const size_t nm = sizeof(uint32_t) * static_cast<size_t>(num_states) * ((s->vocab + 31) / 32);
    TG_CUDA(s->h_mask.ensure(nm));
    TG_CUDA(s->h_state.ensure(sizeof(int32_t) * batch));
    TG_CUDA(cudaMemcpyAsync(s->h_mask.p, mask_table, nm, cudaMemcpyHostToDevice, st));
    TG_CUDA(cudaMemcpyAsync(s->h_state.p, state_id, sizeof(int32_t) * batch, cudaMemcpyHostToDevice, st));
    d_mask = static_cast<const uint32_t*>(s->h_mask.p);
    d_state = static_cast<const int32_t*>(s->h_state.p);
  }
  const float* d_unif = nullptr;
  if (uniforms) {
    TG_CUDA(s->h_unif.ensure(sizeof(float) * batch));
    TG_CUDA(cudaMemcpyAsync(s->h_unif.p, uniforms, sizeof(float) * batch, cudaMemcpyHostToDevice, st));
    d_unif = static_cast<const float*>(s->h_unif.p);
  }
  float* d_prob = nullptr;
  if (out_probs) {
    TG_CUDA(s->h_prob.ensure(sizeof(float) * batch));
    d_prob = static_cast<float*>(s->h_prob.p);
  }
  int32_t rc = tg_sample(s, s->h_logits.p, dtype, row_stride, batch,
                         static_cast<const tg_row_params*>(s->h_params.p), d_hist, d_hlen,
                         history_stride, d_mask, num_states, d_state, d_unif,
                         static_cast<int32_t*>(s->h_out.p), d_prob, st);
  if (rc != TG_OK) return rc;
  TG_CUDA(cudaMemcpyAsync(out_ids, s->h_out.p, sizeof(int32_t) * batch, cudaMemcpyDeviceToHost, st));
  if (out_probs)
    TG_CUDA(cudaMemcpyAsync(out_probs, d_prob, sizeof(float) * batch, cudaMemcpyDeviceToHost, st));
  TG_CUDA(cudaStreamSynchronize(st));
  return TG_OK;
}

static int32_t spec_verify_impl(tg_sampler* s, const void* target_logits, const void* draft_logits,
                                int32_t dtype, int32_t batch, int32_t K, const int32_t* draft_ids,
                                const float* temperature, const float* u_accept, const float* u_draw,
                                const uint32_t* mask_table, int32_t num_states, const int32_t* state_ids,
                                int32_t* out_ids, int32_t* out_n, void* stream) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  if (state_ids && (!mask_table || num_states <= 0))
    return fail(TG_ERR_INVALID_ARG, "state_ids given without mask_table / num_states");
  if (dtype != TG_DTYPE_F32 && dtype != TG_DTYPE_BF16) return fail(TG_ERR_INVALID_ARG, "bad dtype");
  if (batch < 0 || batch > s->max_batch) return fail(TG_ERR_INVALID_ARG, "batch outside [0, max_batch]");
  if (K < 0 || K > 64) return fail(TG_ERR_UNSUPPORTED, "K outside [0, 64]");
  if (batch == 0) return TG_OK;
  if (!target_logits || !temperature || !out_ids || !out_n || (K > 0 && !draft_ids))
    return fail(TG_ERR_INVALID_ARG, "target_logits, draft_ids, temperature, out_ids and out_n are required");
  if (K > 0 && (draft_logits == nullptr) != (u_accept == nullptr))
    return fail(TG_ERR_INVALID_ARG, "draft_logits and u_accept are given together or not at all");
  if (!u_draw) return fail(TG_ERR_INVALID_ARG, "u_draw is required");
  std::lock_guard<std::mutex> lk(s->mu);
  DeviceGuard g(s->device);
  const size_t nst = sizeof(tg::SpecStat) * static_cast<size_t>(batch) * (2 * K + 1);
  if (nst + sizeof(int32_t) * 2 * static_cast<size_t>(batch) > s->stats.cap)
    return fail(TG_ERR_UNSUPPORTED, "verification statistics not reserved for this batch and K (call tg_sampler_reserve)");
  tg::SpecArgs a{target_logits, draft_logits, batch, K, s->vocab, draft_ids, temperature,
                 u_accept, u_draw, out_ids, out_n, static_cast<tg::SpecStat*>(s->stats.p),
                 s->d_status};
  a.rstate = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(s->stats.p) + nst);
  if (state_ids) {
    a.mask_table = mask_table;
    a.num_states = num_states;
    a.mask_words = (s->vocab + 31) / 32;
    a.state_ids = state_ids;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t le = dtype == TG_DTYPE_F32 ? tg::launch_spec<0>(a, st) : tg::launch_spec<1>(a, st);
  if (le == cudaErrorInvalidValue) return fail(TG_ERR_UNSUPPORTED, "vocab too large for the staged verification (vocab * element size > 1.6 MB)");
  TG_CUDA(le);
  return TG_OK;
}

int32_t tg_spec_verify(tg_sampler* s, const void* target_logits, const void* draft_logits,
                       int32_t dtype, int32_t batch, int32_t K, const int32_t* draft_ids,
                       const float* temperature, const float* u_accept, const float* u_draw,
                       int32_t* out_ids, int32_t* out_n, void* stream) {
  return spec_verify_impl(s, target_logits, draft_logits, dtype, batch, K, draft_ids, temperature,
                          u_accept, u_draw, nullptr, 0, nullptr, out_ids, out_n, stream);
}

int32_t tg_spec_verify_masked(tg_sampler* s, const void* target_logits, const void* draft_logits,
                              int32_t dtype, int32_t batch, int32_t K, const int32_t* draft_ids,
                              const float* temperature, const float* u_accept, const float* u_draw,
                              const uint32_t* mask_table, int32_t num_states, const int32_t* state_ids,
                              int32_t* out_ids, int32_t* out_n, void* stream) {
  if (!state_ids) return fail(TG_ERR_INVALID_ARG, "state_ids is required");
  return spec_verify_impl(s, target_logits, draft_logits, dtype, batch, K, draft_ids, temperature,
                          u_accept, u_draw, mask_table, num_states, state_ids, out_ids, out_n, stream);
}

int32_t tg_spec_verify_static(int32_t device, int32_t vocab, const void* target_logits,
                              const void* draft_logits, int32_t dtype, int32_t batch, int32_t K,
                              const int32_t* draft_ids, const float* temperature,
                              const float* u_accept, const float* u_draw, int32_t* out_ids,
                              int32_t* out_n, void* stream) {
  if (dtype != TG_DTYPE_F32 && dtype != TG_DTYPE_BF16) return fail(TG_ERR_INVALID_ARG, "bad dtype");
  if (vocab <= 0 || vocab > TG_MAX_VOCAB) return fail(TG_ERR_UNSUPPORTED, "vocab outside [1, TG_MAX_VOCAB]");
  if (batch < 0 || K < 0 || K > 64) return fail(TG_ERR_INVALID_ARG, "batch < 0 or K outside [0, 64]");
  if (static_cast<int64_t>(batch) * (2 * K + 1) > TG_STATIC_SPEC_MAX_ROWS)
    return fail(TG_ERR_UNSUPPORTED, "batch * (2K + 1) exceeds TG_STATIC_SPEC_MAX_ROWS (the static scratch)");
  if (batch == 0) return TG_OK;
  if (!target_logits || !temperature || !out_ids || !out_n || !u_draw || (K > 0 && !draft_ids))
    return fail(TG_ERR_INVALID_ARG, "missing required pointer");
  if (K > 0 && (draft_logits == nullptr) != (u_accept == nullptr))
    return fail(TG_ERR_INVALID_ARG, "draft_logits and u_accept are given together or not at all");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev || device >= kMaxDevices)
    return fail(TG_ERR_NO_DEVICE, "CUDA device not present");
  DeviceGuard g(device);
  void* scratch = nullptr;
  TG_CUDA(static_scratch(device, &scratch));
  tg::SpecStat* stats = static_cast<tg::SpecStat*>(scratch);
  uint32_t* status = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(scratch) +
                                                 TG_STATIC_SPEC_MAX_ROWS * sizeof(tg::SpecStat));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  TG_CUDA(cudaMemsetAsync(status, 0, sizeof(uint32_t), st));
  tg::SpecArgs a{target_logits, draft_logits, batch, K, vocab, draft_ids, temperature,
                 u_accept, u_draw, out_ids, out_n, stats, status};
  const cudaError_t le = dtype == TG_DTYPE_F32 ? tg::launch_spec<0>(a, st) : tg::launch_spec<1>(a, st);
  if (le == cudaErrorInvalidValue) return fail(TG_ERR_UNSUPPORTED, "vocab too large for the staged verification (vocab * element size > 1.6 MB)");
  TG_CUDA(le);
  return TG_OK;
}

int32_t tg_spec_verify_static_status(int32_t device, uint32_t* out_bits) {
  if (!out_bits) return fail(TG_ERR_INVALID_ARG, "out_bits is NULL");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev || device >= kMaxDevices)
    return fail(TG_ERR_NO_DEVICE, "CUDA device not present");
  DeviceGuard g(device);
  void* scratch = nullptr;
  TG_CUDA(static_scratch(device, &scratch));
  uint32_t* status = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(scratch) +
                                                 TG_STATIC_SPEC_MAX_ROWS * sizeof(tg::SpecStat));
  TG_CUDA(cudaDeviceSynchronize());
  TG_CUDA(cudaMemcpy(out_bits, status, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  TG_CUDA(cudaMemset(status, 0, sizeof(uint32_t)));
  return TG_OK;
}

#ifdef TG_PHASE_TIMING
int32_t tg_debug_phase_cycles(uint64_t* out, int32_t reset) {
  TG_CUDA(cudaDeviceSynchronize());
  TG_CUDA(cudaMemcpyFromSymbol(out, tg::g_phase_cycles, sizeof(uint64_t) * 32));
  if (reset) {
    static const uint64_t z[32] = {};
    TG_CUDA(cudaMemcpyToSymbol(tg::g_phase_cycles, z, sizeof(z)));
  }
  return TG_OK;
}
// per-row phase cycles of rows 0..255 (256 x 16), diagnostic builds only
int32_t tg_debug_row_phases(uint64_t* out, int32_t reset) {
  TG_CUDA(cudaDeviceSynchronize());
  TG_CUDA(cudaMemcpyFromSymbol(out, tg::g_row_phase, sizeof(uint64_t) * 256 * 16));
  if (reset) {
    static const uint64_t z[256 * 16] = {};
    TG_CUDA(cudaMemcpyToSymbol(tg::g_row_phase, z, sizeof(z)));
  }
  return TG_OK;
}
#endif

int32_t tg_sampler_device_status(tg_sampler* s, uint32_t* out_bits) {
  if (!s || !out_bits) return fail(TG_ERR_INVALID_ARG, "NULL argument");
  DeviceGuard g(s->device);
  TG_CUDA(cudaDeviceSynchronize());
  TG_CUDA(cudaMemcpy(out_bits, s->d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  TG_CUDA(cudaMemset(s->d_status, 0, sizeof(uint32_t)));
  return TG_OK;
}

int32_t tg_sampler_path_counters(tg_sampler* s, uint64_t* out, int32_t n, int32_t reset) {
  if (!s || !out || n <= 0) return fail(TG_ERR_INVALID_ARG, "NULL argument or n <= 0");
  DeviceGuard g(s->device);
  TG_CUDA(cudaDeviceSynchronize());
  unsigned long long tmp[TG_PATH_COUNTERS];
  TG_CUDA(cudaMemcpy(tmp, s->d_counters, sizeof(tmp), cudaMemcpyDeviceToHost));
  for (int i = 0; i < n && i < TG_PATH_COUNTERS; i++) out[i] = tmp[i];
  if (reset) TG_CUDA(cudaMemset(s->d_counters, 0, sizeof(tmp)));
  return TG_OK;
}

int32_t tg_sampler_profile(tg_sampler* s, int32_t enable, float* out_ms, int32_t* out_kernels) {
  if (!s) return fail(TG_ERR_INVALID_ARG, "sampler is NULL");
  DeviceGuard g(s->device);
  if (enable && !s->prof_ev[0]) {
    for (cudaEvent_t& ev : s->prof_ev) TG_CUDA(cudaEventCreate(&ev));
  }
  if (out_ms || out_kernels) {
    int n = 0;
    if (s->prof_kind > 0) {
      TG_CUDA(cudaEventSynchronize(s->prof_ev[s->prof_kind]));
      for (int i = 0; i < s->prof_kind; i++) {
        float ms = 0.0f;
        TG_CUDA(cudaEventElapsedTime(&ms, s->prof_ev[i], s->prof_ev[i + 1]));
        if (out_ms) out_ms[i] = ms;
      }
      n = s->prof_kind;
    }
    if (out_kernels) *out_kernels = n;
  }
  s->profile = enable != 0;
  if (!s->profile) s->prof_kind = 0;
  return TG_OK;
}

}  // extern "C"
