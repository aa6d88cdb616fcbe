/*
 * tgsample.h -- C ABI of the B200 batched logits-processing and sampling engine.
 *
 * Drop-in boundary for the sarthak-fleet/tinygpt sampling step: the step that
 * turns the last-position logits of a batch into one token id per row.  Every
 * entry point takes plain pointers and sizes, returns an int32 status
 * (TG_OK = 0, negative on error), never throws and never exits the process.
 * A SwiftPM target binds it through a module map, Python through ctypes.
 *
 * Reference interfaces this ABI replaces (paths are inside sarthak-fleet/tinygpt):
 *   tg_sample        <- TinyGPT.generate sampling block   python_ref/model.py:213-224
 *                    <- tg_generate sampling tail         wasm/src/model.cpp:489-517
 *                       (C ABI declared at wasm/src/model.h:39-43)
 *                    <- sampleToken                       native-mac/Sources/TinyGPTServe/Serve.swift:1483-1506
 *                    <- repetition penalty + top-k        native-mac/Sources/TinyGPTApp/ModelController.swift:262-304
 *                    <- LogitsMasker.mask (as a bitmask)  native-mac/Sources/TinyGPTModel/ConstrainedGen.swift:775-837
 *   tg_spec_verify   <- SpeculativeDecode.stepStochastic  native-mac/Sources/TinyGPT/SpeculativeDecode.swift:121-210
 *                    <- SpeculativeDecode.step (greedy)   native-mac/Sources/TinyGPT/SpeculativeDecode.swift:41-98
 *
 * Memory: all array arguments of tg_sample / tg_spec_verify are DEVICE pointers
 * on the sampler's device, owned by the caller.  The *_host variants take host
 * pointers and stage through buffers the handle owns.  Threading: one handle
 * per device; a handle is not shared between threads without external locking,
 * and serves one stream at a time: its candidate buffer, status word, counters
 * and statistics are per handle, so calls on one handle from two streams that
 * can overlap on the GPU race (use one handle per stream).
 * Allocation: tg_sample allocates nothing (its buffers are made by
 * tg_sampler_create); tg_spec_verify and tg_sample_sharded use buffers made by
 * tg_sampler_reserve and return TG_ERR_UNSUPPORTED for calls beyond them.
 *
 * Semantics (bit-exact definition, restated by the CPU oracle):
 *   y[v]   = logits[v] (bf16 widened exactly to fp32)
 *   penalties, for each distinct id t in the row's history (count c_t):
 *            if repetition_penalty > 1: y = y > 0 ? y / rp : y * rp
 *            if presence or frequency != 0: y = y - (frequency * c_t + presence)
 *   mask   : state_id >= 0 and bit v of mask_table[state_id] clear -> y = -inf
 *   greedy : temperature <= 0 -> first index of max y (-1 if every y is -inf)
 *   s[v]   = y[v] / temperature
 *   top-k  : 0 < top_k < vocab -> keep s >= k-th largest s (ties kept)
 *   mass   : q[v] = trunc(tg_exp(s[v] - max s) * 2^44) as uint64 (exact sums)
 *   top-p  : top_p < 1 -> order survivors by (s desc, id asc), keep the shortest
 *            prefix whose mass reaches top_p * total mass
 *   min-p  : min_p > 0 -> keep q >= min(min_p, 1) * 2^44 (the top survivor has q = 2^44)
 *   draw   : r = trunc(u * S) over the final mass S; first id in INDEX order whose
 *            inclusive running mass exceeds r.
 */
#ifndef TGSAMPLE_H
#define TGSAMPLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------- */
#define TG_OK                 0
#define TG_ERR_INVALID_ARG   -1  /* bad pointer, size, dtype or parameter         */
#define TG_ERR_CUDA          -2  /* a CUDA runtime call failed                    */
#define TG_ERR_UNSUPPORTED   -3  /* size beyond a compiled limit                  */
#define TG_ERR_NO_DEVICE     -4  /* device index not present                      */
#define TG_ERR_DEVICE_STATUS -5  /* a kernel reported a data error (see below)    */
#define TG_ERR_COLLECTIVE    -6  /* a collective missed its deadline; the communicator was aborted */

/* ---- dtypes of the logits --------------------------------------------------- */
#define TG_DTYPE_F32   0
#define TG_DTYPE_BF16  1

/* ---- per-row sampling parameters (32 bytes, POD) ---------------------------
 * temperature <= 0 selects greedy.  top_k <= 0 or >= vocab disables top-k.
 * top_p >= 1 disables top-p.  min_p <= 0 disables min-p.
 * repetition_penalty <= 1 disables the CTRL penalty; presence / frequency
 * penalties of 0 disable them.  flags is reserved and must be 0.            */
typedef struct tg_row_params {
  float   temperature;
  float   top_p;
  float   min_p;
  float   repetition_penalty;
  float   presence_penalty;
  float   frequency_penalty;
  int32_t top_k;
  int32_t flags;
} tg_row_params;

/* Compiled limits. */
#define TG_MAX_VOCAB    (1 << 20)  /* ids must fit in 20 bits                  */
#define TG_MAX_HISTORY  4096       /* history entries per row                  */

typedef struct tg_sampler tg_sampler;

/* Version of this ABI: (major << 16) | minor. */
int32_t tg_abi_version(void);

/* Message for the last error raised on the calling thread ("" if none). */
const char* tg_last_error_string(void);

/* Create a sampler bound to CUDA device `device` for rows of `vocab` logits and
 * at most `max_batch` rows per call.  Allocates the device scratch and the host
 * staging used by the *_host variants; when vocab > 2816 and max_batch >= 1024
 * also the candidate buffer of the two-kernel mode (used for calls of 1024 rows
 * or more), min(max_batch, 2048) rows of
 * 22,536 bytes (46 MB at 2048 rows; environment TG_SAMPLE_SPLIT=0 at creation
 * turns the mode and the buffer off).  Replaces tg_model_create's role as the
 * owner of sampling state (wasm/src/model.h:21-23); returns TG_OK and *out. */
int32_t tg_sampler_create(int32_t device, int32_t vocab, int32_t max_batch,
                          tg_sampler** out);
int32_t tg_sampler_destroy(tg_sampler* s);

/* Sample one token per row.  Device pointers:
 *   logits       [batch, row_stride] of dtype (row_stride >= vocab, in elements)
 *   params       [batch] tg_row_params
 *   history      [batch, history_stride] int32 ids (may be NULL if history_len is NULL)
 *   history_len  [batch] int32, 0..min(history_stride, TG_MAX_HISTORY) (NULL: no history)
 *   mask_table   [num_states, ceil(vocab/32)] uint32, bit set = token allowed (NULL: no masks)
 *   state_id     [batch] int32, -1 = unmasked row (NULL: no masks)
 *   uniforms     [batch] float in [0,1) (ignored for greedy rows)
 *   out_ids      [batch] int32; -1 where no token is admissible
 *   out_probs    [batch] float probability of the chosen id under the final
 *                distribution (1 for greedy rows), may be NULL
 * Asynchronous on `stream` (a cudaStream_t, NULL = legacy default stream);
 * allocates nothing.  The launch shape depends on the batch and never changes
 * a result: 8..148 rows run one 1024-thread CTA per row; 1024 rows or more run
 * two kernels (the stream to the handle's candidate buffer, then selection);
 * other batches run one 256-thread CTA per row.
 * Replaces: python_ref/model.py:213-224, wasm/src/model.cpp:489-517,
 *           Serve.swift:1483-1506, ModelController.swift:262-304. */
int32_t tg_sample(tg_sampler* s, const void* logits, int32_t dtype,
                  int64_t row_stride, int32_t batch, const tg_row_params* params,
                  const int32_t* history, const int32_t* history_len,
                  int32_t history_stride, const uint32_t* mask_table,
                  int32_t num_states, const int32_t* state_id,
                  const float* uniforms, int32_t* out_ids, float* out_probs,
                  void* stream);

/* Same as tg_sample with every array in HOST memory (pinned or pageable).
 * Copies the inputs into the handle's device staging, samples, copies the ids
 * (and probabilities) back and synchronizes before returning.  This is the call
 * a host-side caller with no device memory of its own makes (the Swift serve
 * loop's per-token sampleToken, Serve.swift:1483-1506). */
int32_t tg_sample_host(tg_sampler* s, const void* logits, int32_t dtype,
                       int64_t row_stride, int32_t batch,
                       const tg_row_params* params, const int32_t* history,
                       const int32_t* history_len, int32_t history_stride,
                       const uint32_t* mask_table, int32_t num_states,
                       const int32_t* state_id, const float* uniforms,
                       int32_t* out_ids, float* out_probs);

/* Speculative-decoding verification (rejection sampling), one call per batch.
 * Device pointers:
 *   target_logits [batch, K+1, vocab] of dtype (position K is the bonus position)
 *   draft_logits  [batch, K, vocab] of dtype
 *   draft_ids     [batch, K] int32 proposals
 *   temperature   [batch] float; <= 0 selects greedy verification
 *                 (SpeculativeDecode.swift:41-98), > 0 stochastic with
 *                 T = max(temperature, 1e-5) (SpeculativeDecode.swift:121-210)
 *   u_accept      [batch, K] float uniforms for the accept tests
 *   draft_logits and u_accept may both be NULL (greedy verification without a
 *   draft distribution: Medusa / EAGLE heads, MedusaHeads.swift:186-265,
 *   EagleDraft.swift:216-290); a stochastic row then ends without a token
 *   (out_n = 0) and sets device status bit 4
 *   u_draw        [batch] float uniform for the residual / bonus draw
 *   out_ids       [batch, K+1] int32: accepted proposals then the final token;
 *                 entries past out_n are set to -1
 *   out_n         [batch] int32: number of valid entries (1..K+1)
 * Accept iff u <= min(1, pT(tok) / max(pD(tok), 1e-10)).  On the first reject
 * the final token is drawn from max(0, pT - pD) renormalised when its mass
 * exceeds 1e-10, else from pT; after K accepts it is the bonus drawn from pT at
 * position K.  Probabilities are q / sum(q) with q the exact masses above.
 * Needs statistics reserved by tg_sampler_reserve(s, >= K, ...). */
int32_t tg_spec_verify(tg_sampler* s, const void* target_logits,
                       const void* draft_logits, int32_t dtype, int32_t batch,
                       int32_t K, const int32_t* draft_ids,
                       const float* temperature, const float* u_accept,
                       const float* u_draw, int32_t* out_ids, int32_t* out_n,
                       void* stream);

/* Grammar-masked verification: tg_spec_verify under the constraint of a
 * grammar (mask table as in tg_sample, rows from tg_grammar_state_row).
 * state_ids [batch, K+1] int32 device array: the grammar state before the token
 * of each position (position i's state follows the draft tokens 0..i-1; -1 =
 * unmasked position).  At position i an element whose bit is clear counts as
 * -inf in both the target and the draft rows, so both distributions are
 * renormalised over the allowed tokens, and a disallowed proposal is rejected.
 * A position with no allowed token ends the row without a token (greedy rows:
 * id -1).  A state id >= num_states leaves its position unmasked and sets
 * device status bit 0.  No counterpart in the reference: its speculative paths
 * verify without the grammar mask (docs/constrained_generation.md:243-246). */
int32_t tg_spec_verify_masked(tg_sampler* s, const void* target_logits,
                              const void* draft_logits, int32_t dtype, int32_t batch,
                              int32_t K, const int32_t* draft_ids, const float* temperature,
                              const float* u_accept, const float* u_draw,
                              const uint32_t* mask_table, int32_t num_states,
                              const int32_t* state_ids, int32_t* out_ids, int32_t* out_n,
                              void* stream);

/* Allocation-free variant of tg_spec_verify.  No counterpart in the reference.
 * For callers that cannot call cudaMalloc: for example a serving process that
 * reserved all free HBM for its KV cache at start-up (a cudaMalloc would fail),
 * or a decode loop that must not pay the device-wide synchronization cudaMalloc
 * and cudaFree may cause.  It takes no handle and allocates nothing: the
 * per-position statistics live in a fixed array inside the library, sized for
 * batch * (2K + 1) <= TG_STATIC_SPEC_MAX_ROWS vocab rows (larger calls return
 * TG_ERR_UNSUPPORTED).  Every GPU that loads the library holds that array
 * (about 128 KiB) until the process exits.  The first call on a device looks up
 * the array's device address with that device current; make that first call
 * before any stream capture.  All calls on a device share the array, so calls
 * that overlap on the GPU (different streams without ordering) race.
 * Arguments and results are those of tg_spec_verify, on CUDA device `device`;
 * data errors (bits 1 and 4 of the device status word) are kept in a status
 * word inside the same array, cleared at the start of every call and read by
 * tg_spec_verify_static_status. */
#define TG_STATIC_SPEC_MAX_ROWS 8192
int32_t tg_spec_verify_static(int32_t device, int32_t vocab, const void* target_logits,
                              const void* draft_logits, int32_t dtype, int32_t batch,
                              int32_t K, const int32_t* draft_ids,
                              const float* temperature, const float* u_accept,
                              const float* u_draw, int32_t* out_ids, int32_t* out_n,
                              void* stream);

/* Status bits of the last tg_spec_verify_static call on `device` (meaning as
 * tg_sampler_device_status); synchronizes the device, clears the word,
 * allocates nothing.  No counterpart in the reference. */
int32_t tg_spec_verify_static_status(int32_t device, uint32_t* out_bits);

/* Makes the buffers of the calls that need more than tg_sampler_create's:
 * verification statistics for max_batch rows of up to max_K proposals
 * (tg_spec_verify, tg_spec_verify_masked) and, when max_ranks > 0, the record
 * storage of tg_sample_sharded for communicators of up to max_ranks ranks
 * ((max_ranks + 1) x max_batch x 10,256 bytes).  Buffers only grow.  Call it
 * before the hot loop (and before any stream capture); the hot calls then
 * allocate nothing.  No counterpart in the reference (its C ABI has no
 * device buffers, wasm/src/model.h:39-43). */
int32_t tg_sampler_reserve(tg_sampler* s, int32_t max_K, int32_t max_ranks);

/* ---- vocab-sharded mode (one process per GPU, each owning a vocab slice) ----
 * For vocabularies or batches where one GPU should not hold whole rows: rank r
 * holds ids [vocab_offset, vocab_offset + vocab) of every row (vocab = the
 * handle's vocab).  tg_sample_shard_local writes one record per row: the local
 * survivors of top-k (every local value >= the local k-th, ties kept, global
 * ids) or, for greedy rows, the local first maximum.  The caller all-gathers the
 * records of all ranks (e.g. ncclAllGather / torch.distributed over NVLink) into
 * [nshards][batch] order and every rank calls tg_sample_shard_merge, which
 * returns exactly what tg_sample returns on the whole rows.  Supported rows:
 * greedy, or 0 < top_k <= 1024 (others: id -1 and device status bit 2).
 * No counterpart call exists in the reference (its sampler is single-device);
 * the semantics are those of tg_sample. */
#define TG_SHARD_CAP 1280
typedef struct tg_shard_cand { float value; int32_t id; } tg_shard_cand;
typedef struct tg_shard_record {
  int32_t count;   /* entries in cand; -1: row not supported in sharded mode */
  int32_t flags;   /* bit 0: more than TG_SHARD_CAP local survivors        */
  float absent_max; /* an upper bound of the local values not in cand     */
  int32_t reserved;
  tg_shard_cand cand[TG_SHARD_CAP];
} tg_shard_record;

/* Local half: arguments as tg_sample for this rank's slice (history ids and
 * mask bit positions are global; mask_table rows span full_vocab bits).
 * out_records: [batch] device records. */
int32_t tg_sample_shard_local(tg_sampler* s, int32_t vocab_offset, int32_t full_vocab,
                              const void* logits, int32_t dtype, int64_t row_stride,
                              int32_t batch, const tg_row_params* params,
                              const int32_t* history, const int32_t* history_len,
                              int32_t history_stride, const uint32_t* mask_table,
                              int32_t num_states, const int32_t* state_id,
                              tg_shard_record* out_records, void* stream);

/* Merge half: records [nshards][batch] (gathered), the same params and
 * uniforms on every rank; writes ids / probabilities as tg_sample.  The handle
 * needs max_batch >= batch (its vocab is not used). */
int32_t tg_sample_shard_merge(tg_sampler* s, const tg_shard_record* records, int32_t nshards,
                              int32_t full_vocab, int32_t batch, const tg_row_params* params,
                              const float* uniforms, int32_t* out_ids, float* out_probs,
                              void* stream);

/* Vocab-sharded sampling in one call: the local half (this handle's vocab is the
 * slice [vocab_offset, vocab_offset + vocab) of rows of full_vocab ids), one
 * ncclAllGather of the per-row records over `nccl_comm` (an ncclComm_t of
 * nranks ranks, this rank's slice in rank order), and the merge, all on
 * `stream`; every rank gets the same ids.  Arguments otherwise as tg_sample,
 * for this rank's slice of every row.  NCCL is not linked: ncclAllGather is
 * looked up in the NCCL the process has loaded (TG_ERR_UNSUPPORTED if none).
 * Record storage comes from tg_sampler_reserve(s, ..., >= nranks); nranks must
 * equal the communicator's size (checked with ncclCommCount).  With a collective
 * timeout set (tg_sampler_set_collective_timeout) the call waits on the host for
 * the all-gather and, when it misses the deadline (a rank that left), aborts the
 * communicator (ncclCommAbort) and returns TG_ERR_COLLECTIVE; with none (the
 * default) it only enqueues.  Limits as the two halves
 * (tg_sample_shard_local / tg_sample_shard_merge).  No counterpart in the
 * reference, which samples every row on one device. */
int32_t tg_sample_sharded(tg_sampler* s, void* nccl_comm, int32_t nranks, int32_t vocab_offset,
                          int32_t full_vocab, const void* logits, int32_t dtype, int64_t row_stride,
                          int32_t batch, const tg_row_params* params, const int32_t* history,
                          const int32_t* history_len, int32_t history_stride,
                          const uint32_t* mask_table, int32_t num_states, const int32_t* state_id,
                          const float* uniforms, int32_t* out_ids, float* out_probs, void* stream);

/* Deadline of tg_sample_sharded's all-gather in milliseconds (0: no host wait,
 * the default).  The reference has no collective (single device). */
int32_t tg_sampler_set_collective_timeout(tg_sampler* s, int32_t timeout_ms);

/* Device error word of the last completed call on this handle (synchronizes
 * the handle's device).  Bit 0: a state_id outside [0, num_states);
 * bit 1: a draft id outside [0, vocab); bit 2: a row the vocab-sharded mode
 * could not resolve (unsupported parameters, more than TG_SHARD_CAP local
 * survivors, or a top-k threshold tie between shards); bit 3: a bounded wait
 * of the opt-in fused sampling kernel (TG_FUSED=1) gave up (its rows are
 * unreliable); bit 4: a stochastic row in a verification called without
 * draft logits (it ends without a token).  Cleared by this call. */
int32_t tg_sampler_device_status(tg_sampler* s, uint32_t* out_bits);

/* Per-handle path counters of tg_sample (diagnostics, the device-side analogue
 * of the reference's per-token constraint timing, Serve.swift:1489-1491):
 *   [0] rows finished from the shared-memory candidate list
 *   [1] rows whose candidate list overflowed      -> full-row path
 *   [2] rows with fewer than k candidates         -> full-row path
 *   [3] rows whose top-k threshold fell below the candidate bound -> full-row path
 *   [4] rows processed by the full-row path (any reason)
 *   [5] candidates appended (sum over rows; single-kernel mode)
 *   [6] rows of [0] finished by the warp-group finisher (calls of >= 1024 rows)
 *   [7] rows the warp-group finisher left because its shared-memory pool was full
 * Copies min(n, TG_PATH_COUNTERS) counters (synchronizes the device); zeroes
 * them when reset != 0. */
#define TG_PATH_COUNTERS 8
int32_t tg_sampler_path_counters(tg_sampler* s, uint64_t* out, int32_t n, int32_t reset);

/* Kernel timing of tg_sample (diagnostics): with enable != 0 every later
 * tg_sample call on this handle records CUDA events around its kernels.  Each
 * call of this function first reports the last recorded call (synchronizing on
 * it): *out_kernels = 2 with out_ms[0] the streaming and out_ms[1] the
 * finishing kernel of the two-kernel mode, 1 with out_ms[0] the whole call, 0
 * if none was recorded; then applies `enable`.  out_ms ([2]) and out_kernels
 * may be NULL. */
int32_t tg_sampler_profile(tg_sampler* s, int32_t enable, float* out_ms, int32_t* out_kernels);

/* ---------------------------------------------------------------------------
 * Grammar compiler (host only; no GPU needed): grammar text -> byte-level
 * automaton -> per-state token bitmasks, the rows of tg_sample's mask_table.
 * Replaces the reference's constrained-decoding stack:
 *   ServeGrammarSpec.parse / ServeConstraint / ServeTokenMasker
 *     (native-mac/Sources/TinyGPTServe/Serve.swift:1903-2056),
 *   JSONSchemaNode (native-mac/Sources/TinyGPTModel/JSONSchema.swift:1-117),
 *   JSONSchemaFSM / LogitsMasker (native-mac/Sources/TinyGPTModel/ConstrainedGen.swift:35-837),
 *   PaceToolTagFSM (Serve.swift:2057-2233, grammars/pace-tool-tags.gbnf).
 * Grammar text: after trimming whitespace, text starting with '{' is a JSON
 * Schema (minified JSON only; object keys limited to the declared properties
 * not yet emitted; required keys before '}'; string enum / minLength /
 * maxLength; integer vs number; no trailing commas); a GBNF text holding
 * `root ::=` and `[POINT:` is the tool-tag grammar; anything else is
 * TG_ERR_UNSUPPORTED.
 *
 * Vocabulary: token i is bytes token_bytes[token_offsets[i] .. token_offsets[i+1]).
 * A token is allowed iff the automaton accepts all of its bytes; empty tokens
 * never are.  Once the document is complete only eos_id is allowed (none if
 * eos_id is -1, as in the serve masker). */
#define TG_GRAMMAR_JSON_SCHEMA 0
#define TG_GRAMMAR_TOOL_TAGS 1
typedef struct tg_grammar tg_grammar;
typedef struct tg_grammar_state tg_grammar_state;

const char* tg_grammar_last_error(void);
int32_t tg_grammar_create(const char* grammar_text, int64_t text_len, int32_t vocab,
                          const uint8_t* token_bytes, const int64_t* token_offsets,
                          int32_t eos_id, tg_grammar** out);
int32_t tg_grammar_destroy(tg_grammar* g);
int32_t tg_grammar_kind(tg_grammar* g, int32_t* kind);
/* A fresh automaton at the document start (one per generated sequence). */
int32_t tg_grammar_state_create(tg_grammar* g, tg_grammar_state** out);
int32_t tg_grammar_state_clone(const tg_grammar_state* s, tg_grammar_state** out);
int32_t tg_grammar_state_destroy(tg_grammar_state* s);
/* Feed raw bytes, all or nothing (JSONSchemaFSM.acceptBytes). */
int32_t tg_grammar_accept_bytes(tg_grammar_state* s, const uint8_t* bytes, int64_t n,
                                int32_t* accepted);
/* Advance by a sampled token's bytes (LogitsMasker.commit); *accepted = 0
 * leaves the state unchanged. */
int32_t tg_grammar_commit(tg_grammar_state* s, int32_t token, int32_t* accepted);
int32_t tg_grammar_is_complete(const tg_grammar_state* s, int32_t* out);
/* The state's mask into out_words[ceil(vocab/32)] (bit i%32 of word i/32 = token i). */
int32_t tg_grammar_mask(const tg_grammar_state* s, uint32_t* out_words);
/* The state's row in the grammar's mask table: automaton states with equal
 * futures share a row; the row is computed and appended the first time such a
 * state is seen (*is_new = 1).  The value to put in tg_sample's state_id. */
int32_t tg_grammar_state_row(const tg_grammar_state* s, int32_t* row, int32_t* is_new);
/* The host table (rows x ceil(vocab/32) words, row-major) to upload as
 * tg_sample's mask_table; valid until the next tg_grammar_state_row. */
int32_t tg_grammar_table(tg_grammar* g, const uint32_t** words, int32_t* rows);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* TGSAMPLE_H */
