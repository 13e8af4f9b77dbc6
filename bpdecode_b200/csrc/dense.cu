// Dense regular path: per-state packed allow bits + the per-step mask, commit
// and fused greedy step over bf16 / fp16 / fp32 logits.
//
// Reference semantics: ops.py:262-310 (dense branches of apply_mask_ and
// advance_state), batch.py:176-215 (ConstraintBatch.apply_mask / commit) and
// mask_cpu.cpp:51-90 (step / compute_mask bit layout).
//
// HBM design. A row-step must stream the row of logits once. The allow row of
// a state is 1 bit per token (V/8 bytes, L2-resident: every row in one state
// shares it), read once per 32 tokens by one lane and fanned out with a warp
// shuffle. Each lane owns 16-byte vectors of logits; per vector:
//   all tokens allowed    -> no load, no store (the fused step loads, for argmax)
//   all tokens rejected   -> one 16-byte store of neg_inf, no load
//   mixed                 -> load, blend, store
// so a typical grammar state (almost everything rejected) moves about one
// write of the row instead of a read plus a write.
#include <algorithm>
#include <climits>

#include "common.cuh"
#include "stream.cuh"

namespace bpd {
namespace {

// ---------------------------------------------------------------------------
// Table build (compile time).

__device__ __forceinline__ int32_t dfa_step(const int32_t* __restrict__ trans, int32_t M,
                                            const uint8_t* __restrict__ accept,
                                            const uint8_t* __restrict__ live, int32_t dead,
                                            const int32_t* __restrict__ offsets,
                                            const int32_t* __restrict__ symbols, int32_t eos_id,
                                            int32_t state, int32_t tok) {
  if (tok == eos_id) return accept[state] ? state : -1;
  int32_t cur = state;
  const int32_t end = offsets[tok + 1];
  for (int32_t i = offsets[tok]; i < end; ++i) {
    const int32_t sym = symbols[i];
    if (sym < 0 || sym >= M) return -1;
    cur = trans[static_cast<int64_t>(cur) * M + sym];
    if (cur == dead) return -1;
  }
  return live[cur] ? cur : -1;
}

__global__ void build_tok_next_kernel(const int32_t* __restrict__ trans, int32_t S, int32_t M,
                                      const uint8_t* __restrict__ accept,
                                      const uint8_t* __restrict__ live, int32_t dead,
                                      const int32_t* __restrict__ offsets,
                                      const int32_t* __restrict__ symbols, int32_t V,
                                      int32_t eos_id, const int32_t* __restrict__ rows,
                                      int32_t num_rows, int32_t* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(num_rows) * V;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t r = static_cast<int32_t>(i / V);
    const int32_t t = static_cast<int32_t>(i - static_cast<int64_t>(r) * V);
    const int32_t s = rows ? rows[r] : r;
    out[i] = (s < 0 || s >= S) ? -1
                               : dfa_step(trans, M, accept, live, dead, offsets, symbols, eos_id,
                                          s, t);
  }
}

// One warp builds 32 consecutive words of one state's allow row: 32 coalesced
// 128-byte loads of tok_next, one ballot each.
__global__ void build_allow_bits_kernel(const int32_t* __restrict__ tok_next, int32_t S,
                                        int32_t V, uint32_t* __restrict__ bits, int32_t wstride) {
  const int32_t lane = threadIdx.x & 31;
  const int64_t warp_id = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5;
  const int32_t groups = (wstride + 31) / 32;
  if (warp_id >= static_cast<int64_t>(S) * groups) return;
  const int32_t s = static_cast<int32_t>(warp_id / groups);
  const int32_t w0 = static_cast<int32_t>(warp_id - static_cast<int64_t>(s) * groups) * 32;
  const int32_t* trow = tok_next + static_cast<int64_t>(s) * V;
  uint32_t mine = 0;
  for (int32_t j = 0; j < 32; ++j) {
    const int32_t t = (w0 + j) * 32 + lane;
    const bool ok = (w0 + j) < wstride && t < V && trow[t] != -1;
    const uint32_t b = __ballot_sync(kAll, ok);
    if (lane == j) mine = b;
  }
  if (w0 + lane < wstride) bits[static_cast<int64_t>(s) * wstride + w0 + lane] = mine;
}

__global__ void dense_advance_kernel(int32_t* __restrict__ pool, const int64_t* __restrict__ slots,
                                     int32_t B, const void* __restrict__ tokens, int32_t tokens64,
                                     const int32_t* __restrict__ tok_next, int32_t S, int32_t V,
                                     int32_t* __restrict__ next_out, int32_t write_back) {
  const int32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B) return;
  const int64_t slot = slots ? slots[i] : i;
  const int32_t s = pool[slot];
  const int64_t t = tokens64 ? static_cast<const int64_t*>(tokens)[i]
                             : static_cast<int64_t>(static_cast<const int32_t*>(tokens)[i]);
  const int32_t n = (s < 0 || s >= S || t < 0 || t >= V)
                        ? -1
                        : tok_next[static_cast<int64_t>(s) * V + t];
  if (next_out) next_out[i] = n;
  if (write_back) pool[slot] = n;
}

__global__ void dense_mask_bits_kernel(const int32_t* __restrict__ pool,
                                       const int64_t* __restrict__ slots, int32_t B,
                                       const uint32_t* __restrict__ bits, int32_t wstride,
                                       int32_t S, int32_t W, uint32_t* __restrict__ out) {
  const int32_t row = blockIdx.y;
  int32_t s;
  const uint32_t* brow = state_row(pool, slots, row, bits, wstride, S, &s, nullptr);
  for (int32_t w = blockIdx.x * blockDim.x + threadIdx.x; w < W; w += gridDim.x * blockDim.x)
    out[static_cast<int64_t>(row) * W + w] = brow ? __ldg(brow + w) : 0u;
}

// ---------------------------------------------------------------------------

int esize(int32_t dtype) { return dtype == BPD_F32 ? 4 : 2; }


template <typename T>
bpd_status launch_apply(void* logits, int64_t row_stride, int32_t batch, int32_t V,
                        const int32_t* pool, const int64_t* slots, const uint32_t* bits,
                        int32_t wstride, int32_t S, float neg_inf, cudaStream_t st) {
  return launch_stream_apply<T, DenseRows>(logits, row_stride, batch, V,
                                           DenseRows{pool, slots, bits, wstride, S}, neg_inf, st,
                                           "dense apply kernel");
}

template <typename T>
bpd_status launch_step(void* logits, int64_t row_stride, int32_t batch, int32_t V, int32_t* pool,
                       const int64_t* slots, const uint32_t* bits, int32_t wstride,
                       const int32_t* tok_next, int32_t S, float neg_inf, int64_t* token_out,
                       int32_t* next_out, int32_t chunks_per_row, void* scratch,
                       cudaStream_t st) {
  return launch_stream_step<T, DenseRows, DenseCommit>(
      logits, row_stride, batch, V, DenseRows{pool, slots, bits, wstride, S},
      DenseCommit{pool, tok_next, S, V, token_out, next_out}, neg_inf, chunks_per_row, scratch,
      st, "dense step kernel");
}

}  // namespace
}  // namespace bpd

using namespace bpd;

extern "C" bpd_status bpd_dense_build_tok_next(
    const int32_t* trans, int32_t num_states, int32_t num_symbols, const uint8_t* accept,
    const uint8_t* live, int32_t dead, const int32_t* tok_offsets, const int32_t* tok_symbols,
    int32_t vocab_size, int32_t eos_id, const int32_t* rows, int32_t num_rows,
    int32_t* tok_next_out, void* stream) {
  BPD_REQUIRE(trans && accept && live && tok_offsets && tok_symbols && tok_next_out,
              "bpd_dense_build_tok_next: null pointer");
  BPD_REQUIRE(num_states > 0 && num_symbols > 0 && vocab_size > 0 && num_rows >= 0,
              "bpd_dense_build_tok_next: bad sizes");
  if (num_rows == 0) return BPD_OK;
  const int64_t total = static_cast<int64_t>(num_rows) * vocab_size;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 32);
  build_tok_next_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
      trans, num_states, num_symbols, accept, live, dead, tok_offsets, tok_symbols, vocab_size,
      eos_id, rows, num_rows, tok_next_out);
  return check_launch("build_tok_next_kernel");
}

extern "C" bpd_status bpd_dense_build_allow_bits(const int32_t* tok_next, int32_t num_states,
                                                 int32_t vocab_size, uint32_t* bits_out,
                                                 int32_t words_stride, void* stream) {
  BPD_REQUIRE(tok_next && bits_out, "bpd_dense_build_allow_bits: null pointer");
  BPD_REQUIRE(num_states > 0 && vocab_size > 0, "bpd_dense_build_allow_bits: bad sizes");
  BPD_REQUIRE(words_stride >= (vocab_size + 31) / 32 && words_stride % 4 == 0,
              "bpd_dense_build_allow_bits: words_stride must be >= ceil(vocab/32) and a multiple of 4");
  const int64_t warps = static_cast<int64_t>(num_states) * ((words_stride + 31) / 32);
  const int64_t blocks = (warps * 32 + 255) / 256;
  build_allow_bits_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
      tok_next, num_states, vocab_size, bits_out, words_stride);
  return check_launch("build_allow_bits_kernel");
}

extern "C" bpd_status bpd_dense_apply_mask(void* logits, int32_t dtype, int64_t row_stride,
                                           int32_t batch, int32_t vocab_size,
                                           const int32_t* state_pool, const int64_t* slots,
                                           const uint32_t* allow_bits, int32_t words_stride,
                                           int32_t num_states, float neg_inf, void* stream) {
  BPD_REQUIRE(batch >= 0 && vocab_size > 0, "bpd_dense_apply_mask: bad sizes");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(logits && state_pool && allow_bits, "bpd_dense_apply_mask: null pointer");
  BPD_REQUIRE(row_stride >= vocab_size, "bpd_dense_apply_mask: row_stride < vocab");
  BPD_REQUIRE(words_stride >= (vocab_size + 31) / 32, "bpd_dense_apply_mask: words_stride too small");
  (void)esize;
  cudaStream_t st = as_stream(stream);
  return with_dtype(dtype, "bpd_dense_apply_mask", [&](auto tag) {
    using T = decltype(tag);
    return launch_apply<T>(logits, row_stride, batch, vocab_size, state_pool, slots, allow_bits,
                           words_stride, num_states, neg_inf, st);
  });
}

extern "C" bpd_status bpd_dense_advance(int32_t* state_pool, const int64_t* slots, int32_t batch,
                                        const void* tokens, int32_t tokens_int64,
                                        const int32_t* tok_next, int32_t num_states,
                                        int32_t vocab_size, int32_t* next_out, int32_t write_back,
                                        void* stream) {
  BPD_REQUIRE(batch >= 0 && vocab_size > 0, "bpd_dense_advance: bad sizes");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(state_pool && tokens && tok_next, "bpd_dense_advance: null pointer");
  const int32_t blocks = (batch + 255) / 256;
  dense_advance_kernel<<<blocks, 256, 0, as_stream(stream)>>>(
      state_pool, slots, batch, tokens, tokens_int64, tok_next, num_states, vocab_size, next_out,
      write_back);
  return check_launch("dense_advance_kernel");
}

extern "C" bpd_status bpd_dense_mask_bits(const int32_t* state_pool, const int64_t* slots,
                                          int32_t batch, const uint32_t* allow_bits,
                                          int32_t words_stride, int32_t num_states,
                                          int32_t vocab_size, uint32_t* out_bits, void* stream) {
  BPD_REQUIRE(batch >= 0 && vocab_size > 0, "bpd_dense_mask_bits: bad sizes");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(state_pool && allow_bits && out_bits, "bpd_dense_mask_bits: null pointer");
  BPD_REQUIRE(batch <= 65535, "bpd_dense_mask_bits: batch > 65535");
  const int32_t W = (vocab_size + 31) / 32;
  dim3 grid((W + 255) / 256, batch);
  dense_mask_bits_kernel<<<grid, 256, 0, as_stream(stream)>>>(
      state_pool, slots, batch, allow_bits, words_stride, num_states, W, out_bits);
  return check_launch("dense_mask_bits_kernel");
}

extern "C" size_t bpd_step_scratch_bytes(int32_t batch) {
  return step_scratch_bytes(batch > 0 ? batch : 0);
}

extern "C" bpd_status bpd_dense_step_greedy(void* logits, int32_t dtype, int64_t row_stride,
                                            int32_t batch, int32_t vocab_size, int32_t* state_pool,
                                            const int64_t* slots, const uint32_t* allow_bits,
                                            int32_t words_stride, const int32_t* tok_next,
                                            int32_t num_states, float neg_inf, int64_t* token_out,
                                            int32_t* next_out, int32_t chunks_per_row,
                                            void* step_scratch, void* stream) {
  BPD_REQUIRE(batch >= 0 && vocab_size > 0, "bpd_dense_step_greedy: bad sizes");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(logits && state_pool && allow_bits && tok_next && token_out,
              "bpd_dense_step_greedy: null pointer");
  BPD_REQUIRE(row_stride >= vocab_size, "bpd_dense_step_greedy: row_stride < vocab");
  BPD_REQUIRE(words_stride >= (vocab_size + 31) / 32,
              "bpd_dense_step_greedy: words_stride too small");
  BPD_REQUIRE(chunks_per_row >= 0 && chunks_per_row <= 4096,
              "bpd_dense_step_greedy: chunks_per_row must be in [0, 4096]");
  cudaStream_t st = as_stream(stream);
  return with_dtype(dtype, "bpd_dense_step_greedy", [&](auto tag) {
    using T = decltype(tag);
    return launch_step<T>(logits, row_stride, batch, vocab_size, state_pool, slots, allow_bits,
                          words_stride, tok_next, num_states, neg_inf, token_out, next_out,
                          chunks_per_row, step_scratch, st);
  });
}

extern "C" bpd_status bpd_dense_step_greedy_from(
    const void* src, int32_t src_dtype, int64_t src_stride, const int64_t* src_rows,
    float* out, int64_t out_stride, int32_t batch, int32_t vocab_size, int32_t* state_pool,
    const int64_t* slots, const uint32_t* allow_bits, int32_t words_stride,
    const int32_t* tok_next, int32_t num_states, float neg_inf, int64_t* token_out,
    int32_t* next_out, int32_t chunks_per_row, void* step_scratch, void* stream) {
  BPD_REQUIRE(batch >= 0 && vocab_size > 0, "bpd_dense_step_greedy_from: bad sizes");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(src && state_pool && allow_bits && tok_next && token_out,
              "bpd_dense_step_greedy_from: null pointer");
  BPD_REQUIRE(src_stride >= vocab_size && (out == nullptr || out_stride >= vocab_size),
              "bpd_dense_step_greedy_from: row stride < vocab");
  BPD_REQUIRE(words_stride >= (vocab_size + 31) / 32,
              "bpd_dense_step_greedy_from: words_stride too small");
  BPD_REQUIRE(chunks_per_row >= 0 && chunks_per_row <= 4096,
              "bpd_dense_step_greedy_from: chunks_per_row must be in [0, 4096]");
  cudaStream_t st = as_stream(stream);
  const DenseRows rows{state_pool, slots, allow_bits, words_stride, num_states};
  const DenseCommit commit{state_pool, tok_next, num_states, vocab_size, token_out, next_out};
  const char* what = "bpd_dense_step_greedy_from";
  return with_dtype(src_dtype, what, [&](auto tag) {
    using T = decltype(tag);
    return launch_stream_step_src<T, DenseRows, DenseCommit>(
        src, src_stride, src_rows, out, out_stride, batch, vocab_size, rows, commit, neg_inf,
        chunks_per_row, step_scratch, st, what);
  }, "source");
}
