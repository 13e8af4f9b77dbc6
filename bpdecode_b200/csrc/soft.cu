// Soft lookahead: the k-step backward sum-product table and its per-step
// application (ops.py:200-259).
//
// build: logZ_0(s) = live ? 0 : -inf; k-1 rounds of
//   logZ(s) = live ? LSE_t logZ[tok_next[s,t]] (LSE 0 if s accepts) : -inf
// (the EOS column of tok_next maps an accepting s to itself, so it sits inside
// the sum exactly as in the reference), then out[s,t] = logZ[tok_next[s,t]].
// One CTA per state reduces its row: pass 1 the max (exact), pass 2 the sum of
// expf(x - max) accumulated in double, so the only rounding is one expf per
// term and the final log -- well inside the 1e-5 relative bound against the
// fp32 torch reference. The transition-count formulation (logZ' = log(C e^logZ)
// with C[s, s'] = #tokens s -> s') would make each round an S x S matrix-vector
// product; at S <= ~10^3 and k-1 = 3 rounds it is no contraction worth the
// tensor cores, so the rounds stay a streaming reduction over tok_next.
#include <algorithm>
#include <cfloat>
#include <cmath>

#include "common.cuh"
#include "stream.cuh"

namespace bpd {
namespace {

__global__ void logz_init_kernel(const uint8_t* __restrict__ live, int32_t S, float* __restrict__ logz) {
  const int32_t s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < S) logz[s] = live[s] ? 0.0f : -INFINITY;
}

__device__ __forceinline__ float block_max(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  v = lane < (kThreads / 32) ? sh[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  __syncthreads();
  return v;
}

__device__ __forceinline__ double block_sum(double v, double* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  v = lane < (kThreads / 32) ? sh[lane] : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  __syncthreads();
  return v;
}

__global__ void __launch_bounds__(kThreads)
    lse_round_kernel(const int32_t* __restrict__ tn, int32_t V, const uint8_t* __restrict__ accept,
                     const uint8_t* __restrict__ live, const float* __restrict__ logz_in,
                     float* __restrict__ logz_out) {
  __shared__ float shf[kThreads / 32];
  __shared__ double shd[kThreads / 32];
  const int32_t s = blockIdx.x;
  const int32_t* row = tn + static_cast<int64_t>(s) * V;
  float m = -INFINITY;
  for (int32_t t = threadIdx.x; t < V; t += kThreads) {
    const int32_t n = row[t];
    if (n >= 0) m = fmaxf(m, logz_in[n]);
  }
  m = block_max(m, shf);
  double acc = -INFINITY;
  if (m != -INFINITY) {
    double sum = 0.0;
    for (int32_t t = threadIdx.x; t < V; t += kThreads) {
      const int32_t n = row[t];
      if (n >= 0) sum += static_cast<double>(expf(logz_in[n] - m));
    }
    sum = block_sum(sum, shd);
    acc = static_cast<double>(m) + log(sum);
  }
  if (threadIdx.x == 0) {
    if (accept[s]) {  // logaddexp(acc, 0): EOS from an accepting state reaches DONE
      const double hi = acc > 0.0 ? acc : 0.0;
      acc = (acc == -INFINITY) ? 0.0 : hi + log(exp(acc - hi) + exp(-hi));
    }
    logz_out[s] = live[s] ? static_cast<float>(acc) : -INFINITY;
  }
}

__global__ void lookahead_out_kernel(const int32_t* __restrict__ tn, int32_t S, int32_t V,
                                     const uint8_t* __restrict__ accept, int32_t eos_id,
                                     const float* __restrict__ logz, float* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(S) * V;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t s = static_cast<int32_t>(i / V);
    const int32_t t = static_cast<int32_t>(i - static_cast<int64_t>(s) * V);
    float v;
    if (t == eos_id) {
      v = accept[s] ? 0.0f : -INFINITY;
    } else {
      const int32_t n = tn[i];
      v = n >= 0 ? logz[n] : -INFINITY;
    }
    out[i] = v;
  }
}

// Soft rows: the state picks its allow row (which tiles and vectors are
// live) and its lookahead row (the biases); no state = everything -inf.
struct SoftRows {
  static constexpr bool kSoft = true;
  static constexpr int kTilesPerWarp = BPD_TILES_PER_WARP;
  const int32_t* pool;
  const int64_t* slots;
  const uint32_t* bits;
  int32_t wstride;
  const float* la;
  int32_t S;
  int32_t V;
  float alpha;
  __device__ __forceinline__ RowInfo operator()(int32_t row) const {
    RowInfo r;
    r.brow = state_row(pool, slots, row, bits, wstride, S, &r.state, &r.slot);
    r.lrow = r.brow ? la + static_cast<int64_t>(r.state) * V : nullptr;
    return r;
  }
};

template <typename T>
bpd_status launch_soft_apply(void* logits, int64_t row_stride, int32_t batch, int32_t V,
                             const SoftRows& rows, cudaStream_t st) {
  return launch_stream_apply<T, SoftRows>(logits, row_stride, batch, V, rows, -INFINITY, st,
                                          "bpd_soft_apply");
}

template <typename T>
bpd_status launch_soft_step(void* logits, int64_t row_stride, int32_t batch, int32_t V,
                            const SoftRows& rows, const DenseCommit& commit,
                            int32_t chunks_per_row, void* scratch, cudaStream_t st) {
  return launch_stream_step<T, SoftRows, DenseCommit>(logits, row_stride, batch, V, rows, commit,
                                                      -INFINITY, chunks_per_row, scratch, st,
                                                      "bpd_soft_step_greedy");
}

}  // namespace
}  // namespace bpd

using namespace bpd;

extern "C" size_t bpd_soft_workspace_bytes(int32_t num_states) {
  const size_t b = 2 * sizeof(float) * static_cast<size_t>(num_states > 0 ? num_states : 1);
  return (b + 255) & ~static_cast<size_t>(255);
}

extern "C" bpd_status bpd_soft_build_lookahead(const int32_t* tok_next, int32_t num_states,
                                               int32_t vocab_size, const uint8_t* accept,
                                               const uint8_t* live, int32_t eos_id, int32_t k,
                                               float* out, void* workspace, void* stream) {
  BPD_REQUIRE(tok_next && accept && live && out && workspace,
              "bpd_soft_build_lookahead: null pointer");
  BPD_REQUIRE(num_states > 0 && vocab_size > 0, "bpd_soft_build_lookahead: bad sizes");
  cudaStream_t st = as_stream(stream);
  float* a = static_cast<float*>(workspace);
  float* b = a + num_states;
  logz_init_kernel<<<(num_states + 255) / 256, 256, 0, st>>>(live, num_states, a);
  bpd_status rc = check_launch("logz_init_kernel");
  if (rc) return rc;
  for (int32_t r = 0; r < k - 1; ++r) {
    lse_round_kernel<<<num_states, kThreads, 0, st>>>(tok_next, vocab_size, accept, live, a, b);
    rc = check_launch("lse_round_kernel");
    if (rc) return rc;
    float* t = a;
    a = b;
    b = t;
  }
  const int64_t total = static_cast<int64_t>(num_states) * vocab_size;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 64);
  lookahead_out_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
      tok_next, num_states, vocab_size, accept, eos_id, a, out);
  return check_launch("lookahead_out_kernel");
}

extern "C" bpd_status bpd_soft_apply(void* logits, int32_t dtype, int64_t row_stride,
                                     int32_t batch, int32_t vocab_size, const int32_t* state_pool,
                                     const int64_t* slots, const float* lookahead,
                                     const uint32_t* allow_bits, int32_t words_stride,
                                     int32_t num_states, float alpha, void* stream) {
  BPD_REQUIRE(batch >= 0 && vocab_size > 0, "bpd_soft_apply: bad sizes");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(logits && state_pool && lookahead && allow_bits, "bpd_soft_apply: null pointer");
  BPD_REQUIRE(row_stride >= vocab_size, "bpd_soft_apply: row_stride < vocab");
  BPD_REQUIRE(words_stride >= (vocab_size + 31) / 32, "bpd_soft_apply: words_stride too small");
  cudaStream_t st = as_stream(stream);
  const SoftRows rows{const_cast<int32_t*>(state_pool), slots, allow_bits, words_stride,
                      lookahead, num_states, vocab_size, alpha};
  return with_dtype(dtype, "bpd_soft_apply", [&](auto tag) {
    using T = decltype(tag);
    return launch_soft_apply<T>(logits, row_stride, batch, vocab_size, rows, st);
  });
}

extern "C" bpd_status bpd_soft_step_greedy(void* logits, int32_t dtype, int64_t row_stride,
                                           int32_t batch, int32_t vocab_size, int32_t* state_pool,
                                           const int64_t* slots, const float* lookahead,
                                           const uint32_t* allow_bits, int32_t words_stride,
                                           const int32_t* tok_next, int32_t num_states,
                                           float alpha, int64_t* token_out, int32_t* next_out,
                                           int32_t chunks_per_row, void* step_scratch,
                                           void* stream) {
  BPD_REQUIRE(batch >= 0 && vocab_size > 0, "bpd_soft_step_greedy: bad sizes");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(logits && state_pool && lookahead && allow_bits && tok_next && token_out,
              "bpd_soft_step_greedy: null pointer");
  BPD_REQUIRE(row_stride >= vocab_size, "bpd_soft_step_greedy: row_stride < vocab");
  BPD_REQUIRE(words_stride >= (vocab_size + 31) / 32,
              "bpd_soft_step_greedy: words_stride too small");
  BPD_REQUIRE(chunks_per_row >= 0 && chunks_per_row <= 4096,
              "bpd_soft_step_greedy: chunks_per_row must be in [0, 4096]");
  cudaStream_t st = as_stream(stream);
  const SoftRows rows{state_pool, slots, allow_bits, words_stride, lookahead, num_states,
                      vocab_size, alpha};
  const DenseCommit commit{state_pool, tok_next, num_states, vocab_size, token_out, next_out};
  return with_dtype(dtype, "bpd_soft_step_greedy", [&](auto tag) {
    using T = decltype(tag);
    return launch_soft_step<T>(logits, row_stride, batch, vocab_size, rows, commit,
                               chunks_per_row, step_scratch, st);
  });
}

namespace bpd {
namespace {
bpd_status soft_step_from(
    const void* src, int32_t src_dtype, int64_t src_stride, const int64_t* src_rows,
    float* out, int64_t out_stride, int32_t batch, int32_t vocab_size, int32_t* state_pool,
    const int64_t* slots, const float* lookahead, const uint32_t* allow_bits,
    int32_t words_stride, const int32_t* tok_next, int32_t num_states, float alpha,
    int64_t* token_out, int32_t* next_out, int32_t chunks_per_row, void* step_scratch,
    void* stream, const int32_t* nrows, const char* what) {
  BPD_REQUIRE(batch >= 0 && vocab_size > 0, "%s: bad sizes", what);
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(src && state_pool && lookahead && allow_bits && tok_next && token_out,
              "%s: null pointer", what);
  BPD_REQUIRE(src_stride >= vocab_size && (out == nullptr || out_stride >= vocab_size),
              "%s: row stride < vocab", what);
  BPD_REQUIRE(words_stride >= (vocab_size + 31) / 32,
              "%s: words_stride too small", what);
  BPD_REQUIRE(chunks_per_row >= 0 && chunks_per_row <= 4096,
              "%s: chunks_per_row must be in [0, 4096]", what);
  cudaStream_t st = as_stream(stream);
  const SoftRows rows{state_pool, slots, allow_bits, words_stride, lookahead, num_states,
                      vocab_size, alpha};
  const DenseCommit commit{state_pool, tok_next, num_states, vocab_size, token_out, next_out};
  return with_dtype(src_dtype, what, [&](auto tag) {
    using T = decltype(tag);
    return launch_stream_step_src<T, SoftRows, DenseCommit>(
        src, src_stride, src_rows, out, out_stride, batch, vocab_size, rows, commit, -INFINITY,
        chunks_per_row, step_scratch, st, what, nrows);
  }, "source");
}
}  // namespace
}  // namespace bpd

extern "C" bpd_status bpd_soft_step_greedy_from(
    const void* src, int32_t src_dtype, int64_t src_stride, const int64_t* src_rows,
    float* out, int64_t out_stride, int32_t batch, int32_t vocab_size, int32_t* state_pool,
    const int64_t* slots, const float* lookahead, const uint32_t* allow_bits,
    int32_t words_stride, const int32_t* tok_next, int32_t num_states, float alpha,
    int64_t* token_out, int32_t* next_out, int32_t chunks_per_row, void* step_scratch,
    void* stream) {
  return soft_step_from(src, src_dtype, src_stride, src_rows, out, out_stride, batch, vocab_size,
                        state_pool, slots, lookahead, allow_bits, words_stride, tok_next,
                        num_states, alpha, token_out, next_out, chunks_per_row, step_scratch,
                        stream, nullptr, "bpd_soft_step_greedy_from");
}

extern "C" bpd_status bpd_soft_step_greedy_from_n(
    const void* src, int32_t src_dtype, int64_t src_stride, const int64_t* src_rows,
    float* out, int64_t out_stride, int32_t batch, const int32_t* batch_dev, int32_t vocab_size,
    int32_t* state_pool, const int64_t* slots, const float* lookahead,
    const uint32_t* allow_bits, int32_t words_stride, const int32_t* tok_next,
    int32_t num_states, float alpha, int64_t* token_out, int32_t* next_out,
    int32_t chunks_per_row, void* step_scratch, void* stream) {
  BPD_REQUIRE(batch_dev != nullptr, "bpd_soft_step_greedy_from_n: null row count");
  return soft_step_from(src, src_dtype, src_stride, src_rows, out, out_stride, batch, vocab_size,
                        state_pool, slots, lookahead, allow_bits, words_stride, tok_next,
                        num_states, alpha, token_out, next_out, chunks_per_row, step_scratch,
                        stream, batch_dev, "bpd_soft_step_greedy_from_n");
}
