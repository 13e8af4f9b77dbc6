/*
 * bpdecode_b200 -- C ABI of the B200 (sm_100a) constrained-decoding step.
 *
 * This is the drop-in boundary that replaces bpdecode's torch-op binding
 * (bindings/torch_ops.cpp) and the pure-torch dense path of ops.py. Every
 * entry point takes plain device pointers and sizes -- no torch types -- and
 * enqueues its kernels on `stream` (a cudaStream_t, NULL = legacy default)
 * without synchronising, exactly like the reference ops, which launch on
 * torch's current stream (bindings/torch_ops.cpp:36-42).
 *
 * Errors: every function returns a bpd_status. BPD_OK (0) means the work was
 * enqueued; anything else means nothing was enqueued and bpd_last_error()
 * returns a message for the calling thread. The Python layer turns a non-zero
 * status into RuntimeError, which is what TORCH_CHECK raises in the reference
 * (bindings/torch_ops.cpp:47-51,115-120,301-305,335-339).
 *
 * Layouts (identical to the reference unless marked NEW):
 *   states / state pool  int32, -1 = BROKEN, -2 = FREE (batch.py:31-32)
 *   tok_next             int32 [num_states, vocab] row-major, -1 = reject,
 *                        EOS column = s if s accepts else -1 (ops.py:143-197)
 *   allow bits (NEW)     uint32 [num_states, words_stride], bit t of word t>>5
 *                        set iff tok_next[s,t] != -1 (LSB first, as the
 *                        compute_mask op, mask.hpp:528-531)
 *   PDA config-set       int32 [266] = num_configs, saturated, depth[8],
 *                        stack[8][32] (pda.hpp:82-91)
 *   logits               dtype BPD_F32 / BPD_BF16 / BPD_F16, rows `row_stride`
 *                        elements apart, columns contiguous
 *   slots                optional int64 [batch]: row b reads/writes
 *                        pool[slots[b]]; NULL means row b uses pool[b]
 */
#ifndef BPDECODE_B200_H_
#define BPDECODE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t bpd_status;
#define BPD_OK 0
#define BPD_ERR_INVALID 1   /* bad argument: null pointer, size, dtype, alignment */
#define BPD_ERR_CUDA 2      /* a CUDA runtime call or launch failed */
#define BPD_ERR_CAPACITY 3  /* a size exceeds a documented maximum */

#define BPD_F32 0
#define BPD_BF16 1
#define BPD_F16 2

#define BPD_PDA_MAX_CONFIGS 8
#define BPD_PDA_MAX_DEPTH 32
#define BPD_PDA_CONFIG_INTS (2 + BPD_PDA_MAX_CONFIGS + BPD_PDA_MAX_CONFIGS * BPD_PDA_MAX_DEPTH)

/* NEW (no reference counterpart; the reference reports errors through
 * TORCH_CHECK exceptions, bindings/torch_ops.cpp:47-51): library version. */
const char* bpd_version(void);

/* NEW: message of the last failed call on this host thread ("" if none) --
 * what the reference's TORCH_CHECK message carries. */
const char* bpd_last_error(void);

/* --------------------------------------------------------------------------
 * Dense regular path (regex / non-recursive JSON Schema compiled to a DFA)
 * ------------------------------------------------------------------------ */

/* Dense next-state table from the byte-class DFA: out[r, t] = step(rows[r], t)
 * for every token t (rows == NULL: r = 0..num_rows-1 are the states).
 * Replaces ops.py:143-197 (build_token_transitions); semantics of
 * mask_cpu.cpp:51-67 (step), EOS column as ops.py:190-196. */
bpd_status bpd_dense_build_tok_next(
    const int32_t* trans, int32_t num_states, int32_t num_symbols,
    const uint8_t* accept, const uint8_t* live, int32_t dead,
    const int32_t* tok_offsets, const int32_t* tok_symbols, int32_t vocab_size,
    int32_t eos_id, const int32_t* rows, int32_t num_rows, int32_t* tok_next_out,
    void* stream);

/* NEW: packed allow bits of every tok_next row (bit = tok_next != -1).
 * words_stride >= ceil(vocab/32), a multiple of 4; padding words are zeroed. */
bpd_status bpd_dense_build_allow_bits(
    const int32_t* tok_next, int32_t num_states, int32_t vocab_size,
    uint32_t* bits_out, int32_t words_stride, void* stream);

/* In place: logits[b, t] = neg_inf where state < 0 (BROKEN / FREE), state is
 * out of range, or bit t of the state's allow row is clear. Replaces the dense
 * branch of apply_mask_ (ops.py:271-276) and the apply_mask_ op
 * (bindings/torch_ops.cpp:109-152). neg_inf is rounded to the logits dtype
 * (round to nearest even, as masked_fill_). */
bpd_status bpd_dense_apply_mask(
    void* logits, int32_t dtype, int64_t row_stride, int32_t batch,
    int32_t vocab_size, const int32_t* state_pool, const int64_t* slots,
    const uint32_t* allow_bits, int32_t words_stride, int32_t num_states,
    float neg_inf, void* stream);

/* Commit: next[b] = state < 0 ? -1 : tok_next[state, token[b]] (token out of
 * [0, vocab) -> -1); written to next_out (may be NULL) and, if write_back,
 * into state_pool[slots[b]]. tokens are int32 or int64 (tokens_int64 != 0).
 * Replaces the dense branch of advance_state (ops.py:301-306) and
 * ConstraintBatch.commit's gather/scatter (batch.py:206-215). */
bpd_status bpd_dense_advance(
    int32_t* state_pool, const int64_t* slots, int32_t batch, const void* tokens,
    int32_t tokens_int64, const int32_t* tok_next, int32_t num_states,
    int32_t vocab_size, int32_t* next_out, int32_t write_back, void* stream);

/* Packed allow bits per row, int32 [batch, ceil(vocab/32)] (the compute_mask
 * op, ops.py:284-292 / bindings/torch_ops.cpp:154-189); zero rows for
 * state < 0. */
bpd_status bpd_dense_mask_bits(
    const int32_t* state_pool, const int64_t* slots, int32_t batch,
    const uint32_t* allow_bits, int32_t words_stride, int32_t num_states,
    int32_t vocab_size, uint32_t* out_bits, void* stream);

/* NEW. Device scratch of the fused steps (bpd_dense_step_greedy,
 * bpd_soft_step_greedy) for up to `batch` rows: zero it once before the first
 * call; every call that runs to completion leaves it zero again. One scratch
 * per stream: calls that share it must not run concurrently. */
size_t bpd_step_scratch_bytes(int32_t batch);

/* NEW fused greedy step: apply_mask (as bpd_dense_apply_mask) + argmax of the
 * masked row (first maximal index, NaN counts as maximal, like torch.argmax)
 * + commit of that token (as bpd_dense_advance with write_back = 1).
 * token_out int64 [batch]; next_out int32 [batch] may be NULL.
 * One CTA per (row, chunk); chunks_per_row (0 = automatic, else 1..4096)
 * sets how many chunks a row is cut into. slots may be NULL (row b uses
 * state_pool[b]). step_scratch: bpd_step_scratch_bytes(batch) bytes,
 * 16-byte aligned. */
bpd_status bpd_dense_step_greedy(
    void* logits, int32_t dtype, int64_t row_stride, int32_t batch,
    int32_t vocab_size, int32_t* state_pool, const int64_t* slots,
    const uint32_t* allow_bits, int32_t words_stride, const int32_t* tok_next,
    int32_t num_states, float neg_inf, int64_t* token_out, int32_t* next_out,
    int32_t chunks_per_row, void* step_scratch, void* stream);

/* NEW: the fused step on fp32 working values taken from another buffer --
 * what a caller that upcasts 16-bit model logits to an fp32 copy before
 * masking (hf.py:106-113) gets, without the copy. Row b reads row
 * src_rows[b] of `src` (dtype BPD_F32 / BPD_BF16 / BPD_F16, row stride
 * src_stride; src_rows may be NULL: row b), writes the masked fp32 row to
 * out + b * out_stride (out may be NULL: nothing is written), then the argmax
 * and commit as bpd_dense_step_greedy. `src` is never written. */
bpd_status bpd_dense_step_greedy_from(
    const void* src, int32_t src_dtype, int64_t src_stride, const int64_t* src_rows,
    float* out, int64_t out_stride, int32_t batch, int32_t vocab_size,
    int32_t* state_pool, const int64_t* slots, const uint32_t* allow_bits,
    int32_t words_stride, const int32_t* tok_next, int32_t num_states,
    float neg_inf, int64_t* token_out, int32_t* next_out, int32_t chunks_per_row,
    void* step_scratch, void* stream);

/* --------------------------------------------------------------------------
 * Byte-walk path:/* --------------------------------------------------------------------------
 * Byte-walk path: the same ops on the raw symbol-class DFA, for automata
 * that are not densified (no tok_next table). trans int32 [num_states *
 * num_symbols], accept / live uint8 [num_states], tok_offsets int32 [vocab+1],
 * tok_symbols int32 [tok_offsets[vocab]]; states int32 [batch]. Semantics of
 * mask_cpu.cpp:51-81 (step / compute_mask).
 * ------------------------------------------------------------------------ */

/* In place: logits[b, t] = neg_inf where step(states[b], t) == -1. Replaces
 * the apply_mask_ op's device path (bindings/torch_ops.cpp:109-152,
 * mask_cuda.cu:123-139). batch <= 65535. */
bpd_status bpd_walk_apply_mask(
    void* logits, int32_t dtype, int64_t row_stride, int32_t batch,
    const int32_t* trans, int32_t num_states, int32_t num_symbols,
    const uint8_t* accept, const uint8_t* live, int32_t dead,
    const int32_t* tok_offsets, const int32_t* tok_symbols, int32_t vocab_size,
    int32_t eos_id, const int32_t* states, float neg_inf, void* stream);

/* Packed allow bits int32 [batch, ceil(vocab/32)] (the compute_mask op,
 * bindings/torch_ops.cpp:154-189, mask_cuda.cu:53-80). batch <= 65535. */
bpd_status bpd_walk_mask_bits(
    const int32_t* trans, int32_t num_states, int32_t num_symbols,
    const uint8_t* accept, const uint8_t* live, int32_t dead,
    const int32_t* tok_offsets, const int32_t* tok_symbols, int32_t vocab_size,
    int32_t eos_id, const int32_t* states, int32_t batch, uint32_t* out_bits,
    void* stream);

/* next_out[b] = step(states[b], tokens[b]) (the advance_state op,
 * bindings/torch_ops.cpp:191-229, mask_cuda.cu:106-119). */
bpd_status bpd_walk_advance(
    const int32_t* trans, int32_t num_states, int32_t num_symbols,
    const uint8_t* accept, const uint8_t* live, int32_t dead,
    const int32_t* tok_offsets, const int32_t* tok_symbols, int32_t vocab_size,
    int32_t eos_id, const int32_t* states, const void* tokens, int32_t tokens_int64,
    int32_t batch, int32_t* next_out, void* stream);

/* --------------------------------------------------------------------------
 * Soft lookahead (k-step backward sum-product bias)
 * ------------------------------------------------------------------------ */

/* Lookahead table out[s, t] = logZ_{k-1}(tok_next[s, t]) in fp32, -inf where
 * tok_next = -1, EOS column 0 / -inf by accept. Replaces ops.py:200-236.
 * workspace: at least bpd_soft_workspace_bytes(num_states) bytes. */
size_t bpd_soft_workspace_bytes(int32_t num_states);
bpd_status bpd_soft_build_lookahead(
    const int32_t* tok_next, int32_t num_states, int32_t vocab_size,
    const uint8_t* accept, const uint8_t* live, int32_t eos_id, int32_t k,
    float* out, void* workspace, void* stream);

/* In place: logits += alpha * bias on entries where bias is finite (skipped
 * when alpha == 0), then logits = -inf where bias is -inf; bias =
 * lookahead[state], all -inf for state < 0. Replaces ops.py:239-259.
 * allow_bits / words_stride: the packed allow rows of the same states
 * (bpd_dense_build_allow_bits). A bias is finite only where its token is
 * allowed (true of every table bpd_soft_build_lookahead makes from the same
 * tok_next), so tiles without an allowed token are written without reading
 * the logits or the biases. */
bpd_status bpd_soft_apply(
    void* logits, int32_t dtype, int64_t row_stride, int32_t batch,
    int32_t vocab_size, const int32_t* state_pool, const int64_t* slots,
    const float* lookahead, const uint32_t* allow_bits, int32_t words_stride,
    int32_t num_states, float alpha, void* stream);

/* NEW fused soft step: bpd_soft_apply (with alpha), then the first maximal
 * token of every row (torch.argmax order) into token_out (int64 [batch]) and
 * its commit next = tok_next[state, token] into state_pool[slots[b]] (and
 * next_out, may be NULL). Same results as apply_soft_ + argmax + commit
 * (batch.py:192-215) with one pass over the logits fewer. chunks_per_row and
 * step_scratch as in bpd_dense_step_greedy. */
bpd_status bpd_soft_step_greedy(
    void* logits, int32_t dtype, int64_t row_stride, int32_t batch,
    int32_t vocab_size, int32_t* state_pool, const int64_t* slots,
    const float* lookahead, const uint32_t* allow_bits, int32_t words_stride,
    const int32_t* tok_next, int32_t num_states, float alpha,
    int64_t* token_out, int32_t* next_out, int32_t chunks_per_row,
    void* step_scratch, void* stream);

/* NEW: bpd_soft_step_greedy on fp32 working values read from `src` (the
 * source / destination contract of bpd_dense_step_greedy_from): the biased
 * fp32 rows go to `out` (NULL: not written). */
bpd_status bpd_soft_step_greedy_from(
    const void* src, int32_t src_dtype, int64_t src_stride, const int64_t* src_rows,
    float* out, int64_t out_stride, int32_t batch, int32_t vocab_size,
    int32_t* state_pool, const int64_t* slots, const float* lookahead,
    const uint32_t* allow_bits, int32_t words_stride, const int32_t* tok_next,
    int32_t num_states, float alpha, int64_t* token_out, int32_t* next_out,
    int32_t chunks_per_row, void* step_scratch, void* stream);

/* NEW: bpd_soft_step_greedy_from over the first *batch_dev rows only, where
 * batch_dev (int32, device memory) is read by the kernels, not the host;
 * `batch` is the largest row count the call can see and sizes the launch.
 * The launches do not depend on the row count, so a caller whose mix of
 * requests changes every step (a continuous-batching loop) can replay the
 * step from a CUDA graph. */
bpd_status bpd_soft_step_greedy_from_n(
    const void* src, int32_t src_dtype, int64_t src_stride, const int64_t* src_rows,
    float* out, int64_t out_stride, int32_t batch, const int32_t* batch_dev,
    int32_t vocab_size, int32_t* state_pool, const int64_t* slots,
    const float* lookahead, const uint32_t* allow_bits, int32_t words_stride,
    const int32_t* tok_next, int32_t num_states, float alpha, int64_t* token_out,
    int32_t* next_out, int32_t chunks_per_row, void* step_scratch, void* stream);

/* --------------------------------------------------------------------------
 * Pushdown automaton (context-free grammars)/* --------------------------------------------------------------------------
 * Pushdown automaton (context-free grammars)
 * ------------------------------------------------------------------------ */

/* The flattened grammar + token bytes (grammar/device.py:33-76): plain
 * device pointers, as the reference's PdaTableView (pda_cuda.cu:22-33). */
typedef struct bpd_pda_grammar {
  int32_t num_states;
  int32_t num_edges;
  int32_t root_start;
  int32_t root_accept;
  const uint8_t* accept;        /* [num_states] */
  const uint8_t* live;          /* [num_states] */
  const int32_t* edge_offsets;  /* [num_states + 1] */
  const int32_t* edge_kind;     /* [num_edges] 0 eps, 1 byte range, 2 call */
  const int32_t* edge_lo;       /* [num_edges] */
  const int32_t* edge_hi;       /* [num_edges] */
  const int32_t* edge_dst;      /* [num_edges] */
  const int32_t* edge_callee;   /* [num_edges] */
  int32_t vocab_size;
  int32_t eos_id;               /* -1: none */
  const int32_t* tok_offsets;   /* [vocab_size + 1] */
  const uint8_t* tok_bytes;     /* [tok_offsets[vocab_size]] */
} bpd_pda_grammar;

/* Initial config-set (pda.hpp:200-207) into config_out[266], on the device.
 * Replaces the host pda_init op (bindings/torch_ops.cpp:307-324). */
bpd_status bpd_pda_init(const bpd_pda_grammar* g, int32_t* config_out, void* stream);

/* Mask-memo table in caller-owned device memory (NEW; the per-config mask memo
 * held in HBM). bpd_pda_memo_bytes gives the size for `capacity` entries;
 * bpd_pda_memo_reset clears it (call once after allocating, and to drop every
 * cached mask). capacity must be a power of two; the buffer 16-byte aligned.
 * It also holds the miss path's transition cache (16 config-set nodes per
 * entry); a call that finds that cache full has the next call start it over.
 * Calls that share a memo must be ordered on one stream; after a call that
 * failed on the device, reset the memo before using it again. */
size_t bpd_pda_memo_bytes(int32_t capacity, int32_t vocab_size);
bpd_status bpd_pda_memo_reset(void* memo, int32_t capacity, int32_t vocab_size,
                              void* stream);

/* NEW: per-call scratch of bpd_pda_apply_mask / bpd_pda_mask_bits /
 * bpd_pda_step_greedy for `batch` rows (the reference allocates its per-row
 * PdaConfigSet copies in local memory inside its kernels, pda_cuda.cu:40-95).
 * 16-byte aligned; any contents (each call clears what it needs). */
size_t bpd_pda_workspace_bytes(int32_t batch, int32_t vocab_size);

/* Packed allow bits per row, int32 [batch, ceil(vocab/32)], of config-set
 * pool[slots[b]] (compute_mask_pda_batch, pda_cpu.cpp:7-21). memo may be NULL
 * (no caching). Rows whose broken flag is set (broken may be NULL) get zeros. */
bpd_status bpd_pda_mask_bits(
    const bpd_pda_grammar* g, const int32_t* config_pool, const int64_t* slots,
    const uint8_t* broken, int32_t batch, void* memo, int32_t memo_capacity,
    void* workspace, uint32_t* out_bits, void* stream);

/* In place: logits[b, t] = neg_inf where token t is rejected from config-set
 * pool[slots[b]] (pda_try_token, pda.hpp:248-258; EOS allowed iff complete)
 * and on every column of rows whose broken flag is set. Replaces the
 * pda_apply_mask_ op (bindings/torch_ops.cpp:326-376) plus the broken-row fill
 * of CFGConstraintBatch.apply_mask (grammar/device.py:252-266), without the
 * host sync. Any logits dtype. */
bpd_status bpd_pda_apply_mask(
    const bpd_pda_grammar* g, void* logits, int32_t dtype, int64_t row_stride,
    const int32_t* config_pool, const int64_t* slots, const uint8_t* broken,
    int32_t batch, void* memo, int32_t memo_capacity, void* workspace,
    float neg_inf, void* stream);

/* NEW fused greedy step of the PDA path: bpd_pda_apply_mask, then the first
 * maximal token of every masked row (torch.argmax order) into token_out
 * (int64 [batch]), then bpd_pda_advance of those tokens (broken / status_out
 * as there; broken may be NULL). Identical results to apply_mask + argmax +
 * commit (grammar/device.py:252-283) with one pass over the logits fewer.
 * chunks_per_row as in bpd_dense_step_greedy; the step's scratch lives in
 * the workspace (bpd_pda_workspace_bytes). */
bpd_status bpd_pda_step_greedy(
    const bpd_pda_grammar* g, void* logits, int32_t dtype, int64_t row_stride,
    int32_t* config_pool, const int64_t* slots, uint8_t* broken, int32_t batch,
    void* memo, int32_t memo_capacity, void* workspace, float neg_inf,
    int64_t* token_out, int32_t* status_out, int32_t chunks_per_row, void* stream);

/* NEW: bpd_pda_step_greedy on fp32 working values read from `src` (the
 * source / destination contract of bpd_dense_step_greedy_from); the reference
 * PDA op takes fp32 logits only (torch_ops.cpp:334-335), which callers with
 * 16-bit logits meet by upcasting a copy. */
bpd_status bpd_pda_step_greedy_from(
    const bpd_pda_grammar* g, const void* src, int32_t src_dtype,
    int64_t src_stride, const int64_t* src_rows, float* out, int64_t out_stride,
    int32_t* config_pool, const int64_t* slots, uint8_t* broken, int32_t batch,
    void* memo, int32_t memo_capacity, void* workspace, float neg_inf,
    int64_t* token_out, int32_t* status_out, int32_t chunks_per_row, void* stream);

/* NEW: bpd_pda_step_greedy_from over the first *batch_dev rows only (int32
 * in device memory, read by the kernels; `batch` bounds it and sizes the
 * launches and the workspace), as bpd_soft_step_greedy_from_n. */
bpd_status bpd_pda_step_greedy_from_n(
    const bpd_pda_grammar* g, const void* src, int32_t src_dtype,
    int64_t src_stride, const int64_t* src_rows, float* out, int64_t out_stride,
    int32_t* config_pool, const int64_t* slots, uint8_t* broken, int32_t batch,
    const int32_t* batch_dev, void* memo, int32_t memo_capacity, void* workspace,
    float neg_inf, int64_t* token_out, int32_t* status_out, int32_t chunks_per_row,
    void* stream);

/* --------------------------------------------------------------------------
 * Continuous-batching turnover on the device (NEW; the reference leaves the
 * serving loop to its callers, vllm.py:100-184). A loop of `rows` rows holds
 * one request per row: kind[row] 0 = a dense-grammar request (DFA state in
 * state_pool[row]), 1 = a PDA request (config_pool[row], broken[row]); row r
 * uses slot r of both pools. dense_rows / pda_rows (int64 [rows]) list the
 * rows of each kind in ascending order, counts (int32 [2]) their lengths --
 * the row lists and device row counts of the *_from_n steps.
 * ------------------------------------------------------------------------ */

/* Retire and admit requests: row r retires with probability evict_prob, drawn
 * from a counter-based hash of (seed, *step_counter, r) (uint64 counter in
 * device memory, advanced by one per call). A retired row's new request is a
 * regex (dense grammar uniform in [0, n_regex)) with probability p_regex, the
 * dense grammar schema_grammar (-1: none) with probability p_schema, else a
 * PDA request; its state starts at dense_starts[grammar] (int32, device), or
 * its config-set at pda_init (int32 [BPD_PDA_CONFIG_INTS], device) with
 * broken cleared (a PDA row's dense state becomes FREE, -2). retired (uint8
 * [rows]) records which rows turned over; the row lists and counts are
 * rebuilt. One CTA; any `rows`. */
bpd_status bpd_serving_turnover(
    int32_t rows, uint64_t seed, uint64_t* step_counter, float evict_prob,
    float p_regex, float p_schema, int32_t n_regex, int32_t schema_grammar,
    const int32_t* dense_starts, const int32_t* pda_init, int32_t* kind,
    int32_t* state_pool, int32_t* config_pool, uint8_t* broken,
    int64_t* dense_rows, int64_t* pda_rows, int32_t* counts, uint8_t* retired,
    void* stream);

/* tokens_out[dense_rows[b]] = dense_tok[b] for b < counts[0] and
 * tokens_out[pda_rows[b]] = pda_tok[b] for b < counts[1]: the two steps'
 * tokens back in row order (int64). */
bpd_status bpd_serving_gather_tokens(
    int32_t rows, const int64_t* dense_rows, const int64_t* pda_rows,
    const int32_t* counts, const int64_t* dense_tok, const int64_t* pda_tok,
    int64_t* tokens_out, void* stream);

/* Advance config-set pool[slots[b]] in place by tokens[b] (int32 or int64)./* Advance config-set pool[slots[b]] in place by tokens[b] (int32 or int64).
 * ok_out[b] (uint8, may be NULL) = 1 if the token was accepted; a rejected
 * token leaves the config-set unchanged; EOS sets ok = complete and never
 * changes it (pda_cpu.cpp:35-54). If broken != NULL: broken[slot] |= !ok, and
 * status_out[b] (int32, may be NULL) = broken[slot] ? -1 : 1
 * (grammar/device.py:268-283). Replaces the pda_advance_state op
 * (bindings/torch_ops.cpp:378-425). */
bpd_status bpd_pda_advance(
    const bpd_pda_grammar* g, int32_t* config_pool, const int64_t* slots,
    int32_t batch, const void* tokens, int32_t tokens_int64, uint8_t* ok_out,
    uint8_t* broken, int32_t* status_out, void* stream);

/* Allocation-free form of bpd_pda_apply_mask, for callers that cannot
 * allocate device memory at the point they mask: a serving engine that has
 * handed (nearly) all of HBM to its own pool or KV cache, so a raw cudaMalloc
 * would fail or fragment that pool, or a foreign-language binding (ctypes,
 * FFI) that has no access to the host framework's allocator. No counterpart in
 * the reference. Same arguments and results as bpd_pda_apply_mask minus the
 * workspace: the per-call scratch is a fixed device array built into this
 * library, sized for at most BPD_NOALLOC_MAX_BATCH rows of at most
 * BPD_NOALLOC_MAX_VOCAB tokens (about 4.2 MB, held on every device that loads
 * the library until exit); larger calls fail with BPD_ERR_CAPACITY. memo may
 * be NULL (no mask caching). Nothing here calls cudaMalloc or cudaFree.
 * The first call on a device looks up the array's device address (once per
 * device, with that device current); make that first call before any stream
 * capture. The address is kept with the driver context it belongs to: after
 * cudaDeviceReset the next call looks it up again in the new context (so that
 * call, too, should come before any capture). All calls share the one array, so calls that can overlap on the
 * GPU (different streams, different host threads) race on it: serialise them
 * on one stream. Each call clears what it needs zeroed itself. */
#define BPD_NOALLOC_MAX_BATCH 128
#define BPD_NOALLOC_MAX_VOCAB 262144
bpd_status bpd_pda_apply_mask_noalloc(
    const bpd_pda_grammar* g, void* logits, int32_t dtype, int64_t row_stride,
    const int32_t* config_pool, const int64_t* slots, const uint8_t* broken,
    int32_t batch, void* memo, int32_t memo_capacity, float neg_inf, void* stream);

/* complete_out[b] (uint8) = pda_is_complete(pool[slots[b]]) && !broken
 * (pda.hpp:238-244; CFGConstraintBatch.is_complete, grammar/device.py:286-297). */
bpd_status bpd_pda_is_complete(
    const bpd_pda_grammar* g, const int32_t* config_pool, const int64_t* slots,
    const uint8_t* broken, int32_t batch, uint8_t* complete_out, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* BPDECODE_B200_H_ */
