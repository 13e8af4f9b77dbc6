// Byte-walk path: the reference's apply_mask_ / compute_mask / advance_state
// ops on the raw symbol-class DFA (trans / offsets / symbols) when no dense
// tok_next table exists -- automata too large to densify, or callers of the
// torch.ops.bpdecode.* schemas (bindings/torch_ops.cpp:109-229).
//
// Semantics of mask_cpu.cpp:51-81 (step / compute_mask). Each thread walks one
// (row, token) pair; a CTA owns a block of 256 tokens of one row, so a warp's
// 32 verdicts are one ballot = one allow word. The transition table is staged
// in shared memory when it fits (regexes: a few hundred entries), otherwise
// read through L1.
#include <algorithm>

#include "common.cuh"

namespace bpd {
namespace {

constexpr int kWalkThreads = 256;
constexpr int32_t kSmemTrans = 8192;  // int32 entries staged per CTA (32 KB)

__device__ __forceinline__ int32_t walk_step(const int32_t* __restrict__ trans, int32_t M,
                                             const uint8_t* __restrict__ accept,
                                             const uint8_t* __restrict__ live, int32_t dead,
                                             int32_t S, const int32_t* __restrict__ offsets,
                                             const int32_t* __restrict__ symbols, int32_t eos_id,
                                             int32_t state, int32_t tok) {
  if (tok == eos_id) return (state >= 0 && state < S && __ldg(accept + state)) ? state : -1;
  if (state < 0 || state >= S) return -1;
  int32_t cur = state;
  const int32_t end = __ldg(offsets + tok + 1);
  for (int32_t i = __ldg(offsets + tok); i < end; ++i) {
    const int32_t sym = __ldg(symbols + i);
    if (sym < 0 || sym >= M) return -1;
    cur = trans[static_cast<int64_t>(cur) * M + sym];
    if (cur == dead) return -1;
    if (cur < 0 || cur >= S) return -1;
  }
  return __ldg(live + cur) ? cur : -1;
}

struct WalkDfa {
  const int32_t* trans;
  const uint8_t* accept;
  const uint8_t* live;
  const int32_t* offsets;
  const int32_t* symbols;
  int32_t S, M, dead, V, eos_id;
};

// grid: (ceil(V / 256), batch). Writes neg_inf into rejected logits (logits
// != nullptr) and/or the packed allow words (bits != nullptr).
template <typename T>
__global__ void __launch_bounds__(kWalkThreads)
    walk_mask_kernel(WalkDfa d, const int32_t* __restrict__ states, T* __restrict__ logits,
                     int64_t row_stride, typename Dt<T>::Bits fill, uint32_t* __restrict__ bits,
                     int32_t words) {
  __shared__ int32_t strans[kSmemTrans];
  const int64_t n = static_cast<int64_t>(d.S) * d.M;
  const int32_t* trans = d.trans;
  if (n <= kSmemTrans) {
    for (int32_t i = threadIdx.x; i < n; i += kWalkThreads) strans[i] = __ldg(d.trans + i);
    __syncthreads();
    trans = strans;
  }
  const int32_t row = blockIdx.y;
  const int32_t t = blockIdx.x * kWalkThreads + threadIdx.x;
  const int32_t s = states[row];
  const bool ok = t < d.V &&
                  walk_step(trans, d.M, d.accept, d.live, d.dead, d.S, d.offsets, d.symbols,
                            d.eos_id, s, t) != -1;
  if (logits && t < d.V && !ok) {
    reinterpret_cast<typename Dt<T>::Bits*>(logits + row * row_stride)[t] = fill;
  }
  if (bits) {
    const uint32_t w = __ballot_sync(0xFFFFFFFFu, ok);
    const int32_t word = (blockIdx.x * kWalkThreads + (threadIdx.x & ~31)) >> 5;
    if ((threadIdx.x & 31) == 0 && word < words) bits[static_cast<int64_t>(row) * words + word] = w;
  }
}

__global__ void walk_advance_kernel(WalkDfa d, const int32_t* __restrict__ states,
                                    const void* __restrict__ tokens, int32_t tokens64,
                                    int32_t batch, int32_t* __restrict__ next) {
  const int32_t b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int64_t t = tokens64 ? static_cast<const int64_t*>(tokens)[b]
                             : static_cast<int64_t>(static_cast<const int32_t*>(tokens)[b]);
  next[b] = (t < 0 || t >= d.V) ? -1
                                : walk_step(d.trans, d.M, d.accept, d.live, d.dead, d.S, d.offsets,
                                            d.symbols, d.eos_id, states[b],
                                            static_cast<int32_t>(t));
}

bpd_status check_dfa(const WalkDfa& d, const char* what) {
  if (!(d.trans && d.accept && d.live && d.offsets && d.symbols))
    return fail(BPD_ERR_INVALID, "%s: null table pointer", what);
  if (d.S <= 0 || d.M <= 0 || d.V <= 0) return fail(BPD_ERR_INVALID, "%s: bad sizes", what);
  return BPD_OK;
}

template <typename T>
bpd_status launch_walk_mask(const WalkDfa& d, const int32_t* states, int32_t batch, void* logits,
                            int64_t row_stride, float neg_inf, uint32_t* bits, cudaStream_t st) {
  dim3 grid((d.V + kWalkThreads - 1) / kWalkThreads, batch);
  walk_mask_kernel<T><<<grid, kWalkThreads, 0, st>>>(
      d, states, static_cast<T*>(logits), row_stride, Dt<T>::from_float_host(neg_inf), bits,
      (d.V + 31) / 32);
  return check_launch("walk_mask_kernel");
}

}  // namespace
}  // namespace bpd

using namespace bpd;

extern "C" bpd_status bpd_walk_apply_mask(void* logits, int32_t dtype, int64_t row_stride,
                                          int32_t batch, const int32_t* trans, int32_t num_states,
                                          int32_t num_symbols, const uint8_t* accept,
                                          const uint8_t* live, int32_t dead,
                                          const int32_t* tok_offsets, const int32_t* tok_symbols,
                                          int32_t vocab_size, int32_t eos_id,
                                          const int32_t* states, float neg_inf, void* stream) {
  const WalkDfa d{trans, accept, live, tok_offsets, tok_symbols,
                  num_states, num_symbols, dead, vocab_size, eos_id};
  bpd_status rc = check_dfa(d, "bpd_walk_apply_mask");
  if (rc) return rc;
  BPD_REQUIRE(batch >= 0 && batch <= 65535, "bpd_walk_apply_mask: batch out of range");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(logits && states, "bpd_walk_apply_mask: null pointer");
  BPD_REQUIRE(row_stride >= vocab_size, "bpd_walk_apply_mask: row_stride < vocab");
  cudaStream_t st = as_stream(stream);
  return with_dtype(dtype, "bpd_walk_apply_mask", [&](auto tag) {
    using T = decltype(tag);
    return launch_walk_mask<T>(d, states, batch, logits, row_stride, neg_inf, nullptr, st);
  });
}

extern "C" bpd_status bpd_walk_mask_bits(const int32_t* trans, int32_t num_states,
                                         int32_t num_symbols, const uint8_t* accept,
                                         const uint8_t* live, int32_t dead,
                                         const int32_t* tok_offsets, const int32_t* tok_symbols,
                                         int32_t vocab_size, int32_t eos_id,
                                         const int32_t* states, int32_t batch,
                                         uint32_t* out_bits, void* stream) {
  const WalkDfa d{trans, accept, live, tok_offsets, tok_symbols,
                  num_states, num_symbols, dead, vocab_size, eos_id};
  bpd_status rc = check_dfa(d, "bpd_walk_mask_bits");
  if (rc) return rc;
  BPD_REQUIRE(batch >= 0 && batch <= 65535, "bpd_walk_mask_bits: batch out of range");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(states && out_bits, "bpd_walk_mask_bits: null pointer");
  return launch_walk_mask<float>(d, states, batch, nullptr, 0, 0.0f, out_bits,
                                 as_stream(stream));
}

extern "C" bpd_status bpd_walk_advance(const int32_t* trans, int32_t num_states,
                                       int32_t num_symbols, const uint8_t* accept,
                                       const uint8_t* live, int32_t dead,
                                       const int32_t* tok_offsets, const int32_t* tok_symbols,
                                       int32_t vocab_size, int32_t eos_id, const int32_t* states,
                                       const void* tokens, int32_t tokens_int64, int32_t batch,
                                       int32_t* next_out, void* stream) {
  const WalkDfa d{trans, accept, live, tok_offsets, tok_symbols,
                  num_states, num_symbols, dead, vocab_size, eos_id};
  bpd_status rc = check_dfa(d, "bpd_walk_advance");
  if (rc) return rc;
  BPD_REQUIRE(batch >= 0, "bpd_walk_advance: bad batch");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(states && tokens && next_out, "bpd_walk_advance: null pointer");
  walk_advance_kernel<<<(batch + 255) / 256, 256, 0, as_stream(stream)>>>(
      d, states, tokens, tokens_int64, batch, next_out);
  return check_launch("walk_advance_kernel");
}
