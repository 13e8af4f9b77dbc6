// Request turnover of a continuous-batching serving loop, on the device.
//
// A loop over `rows` rows holds one request per row; a request is either a
// dense-grammar request (its DFA state in state_pool[row]) or a PDA request
// (its config-set in config_pool[row], its broken flag in broken[row]). Row r
// always uses slot r of both pools. Each step the loop runs the fused dense
// step over the rows listed in dense_rows[0, counts[0]) and the fused PDA step
// over pda_rows[0, counts[1]); both read their row counts from device memory,
// so a step has the same launches whatever the mix and can be replayed from a
// CUDA graph. After the step:
//
// * bpd_serving_gather_tokens puts each list's tokens back in row order;
// * bpd_serving_turnover retires requests and admits new ones in their rows:
//   row r retires with probability evict_prob (a counter-based hash of
//   (seed, step, r), so a run is reproducible and independent of timing), the
//   new request is a regex (grammar uniform in [0, n_regex)) with probability
//   p_regex, the schema grammar `schema_grammar` with probability p_schema,
//   else a PDA request; its state / config-set starts fresh; then the two row
//   lists and counts are rebuilt and the step counter advances.
//
// The hash is SplitMix64's output function (Steele, Lea, Flood 2014) over
// seed ^ (step * golden-ratio increment) ^ (row, stream) words.
#include "common.cuh"

namespace bpd {
namespace {

constexpr int kTurnThreads = 1024;
constexpr int NCFG = BPD_PDA_CONFIG_INTS;

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Uniform in [0, 1) with 24 bits, from (seed, step, row, stream).
__device__ __forceinline__ float unit_draw(uint64_t seed, uint64_t step, int32_t row,
                                           uint32_t stream) {
  const uint64_t h = splitmix64(seed ^ splitmix64(step * 0x9E3779B97F4A7C15ull ^
                                                  (static_cast<uint64_t>(row) << 8 | stream)));
  return static_cast<float>(h >> 40) * (1.0f / 16777216.0f);
}

struct TurnArgs {
  int32_t rows;
  uint64_t seed;
  uint64_t* step;  // device counter
  float evict_prob, p_regex, p_schema;
  int32_t n_regex, schema_grammar;
  const int32_t* dense_starts;
  const int32_t* pda_init;
  int32_t* kind;
  int32_t* state_pool;
  int32_t* config_pool;
  uint8_t* broken;
  int64_t* dense_rows;
  int64_t* pda_rows;
  int32_t* counts;
  uint8_t* retired;
};

// One CTA of 1024 threads; thread t handles rows t, t + 1024, ... in every
// phase. Phase 1: draw, retire, write the new kind and dense state; the
// thread keeps its rows' kinds (up to kRowsInRegs rows a thread) for phase 3,
// and admitted PDA rows go to a shared list. Phase 2 (a warp per listed row):
// the fresh config-sets. Phase 3: the row lists, an order-preserving
// compaction (ballot + warp prefix sums + a running base per 1024 rows).
constexpr int kRowsInRegs = 8;       // rows up to 8192 keep their kinds in registers
constexpr int kAdmitList = 2048;     // admitted PDA rows listed in shared memory
constexpr int kStartsInSmem = 64;    // dense grammars whose start state is staged

__global__ void __launch_bounds__(kTurnThreads) turnover_kernel(TurnArgs a) {
  __shared__ int32_t warp_d[kTurnThreads / 32], warp_p[kTurnThreads / 32];
  __shared__ int32_t base_d, base_p, n_admit;
  __shared__ int32_t admit[kAdmitList];
  __shared__ int32_t init_s[NCFG];
  __shared__ int32_t starts_s[kStartsInSmem];
  const int32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    base_d = 0;
    base_p = 0;
    n_admit = 0;
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // kinds, pools and lists are the step kernels' until they end
  // every load below is issued before the first one is waited for: the step
  // counter, each thread's first kind, the fresh config-set and the dense
  // grammars' start states (-4.5 us on the config-5 serving step)
  const uint64_t step = *a.step;
  if (tid < NCFG) init_s[tid] = a.pda_init[tid];
  const int32_t nstarts = max(a.n_regex, a.schema_grammar + 1);
  if (tid < nstarts && tid < kStartsInSmem) starts_s[tid] = a.dense_starts[tid];
  int32_t was = tid < a.rows ? a.kind[tid] : 0;
  __syncthreads();
  int32_t kinds[kRowsInRegs];
#pragma unroll
  for (int j = 0; j < kRowsInRegs; ++j) kinds[j] = -1;
  for (int32_t r = tid, j = 0; r < a.rows; r += kTurnThreads, ++j) {
    if (j > 0) was = a.kind[r];
    const bool out = unit_draw(a.seed, step, r, 0) < a.evict_prob;
    int32_t k = out ? 1 : was;
    a.retired[r] = out ? 1 : 0;
    if (out) {
      const float u = unit_draw(a.seed, step, r, 1);
      int32_t g = -1;
      if (u < a.p_regex) {
        k = 0;
        g = min(a.n_regex - 1, static_cast<int32_t>(unit_draw(a.seed, step, r, 2) *
                                                    static_cast<float>(a.n_regex)));
      } else if (a.schema_grammar >= 0 && u < a.p_regex + a.p_schema) {
        k = 0;
        g = a.schema_grammar;
      }
      a.kind[r] = k;
      if (k == 0) {
        a.state_pool[r] = g < kStartsInSmem ? starts_s[g] : a.dense_starts[g];
      } else {
        a.state_pool[r] = -2;  // FREE for a PDA request
      }
      if (k == 1) {
        a.broken[r] = 0;
        const int32_t at = atomicAdd(&n_admit, 1);
        if (at < kAdmitList) admit[at] = r;
      }
    }
    if (j < kRowsInRegs) kinds[j] = k;
  }
  __syncthreads();
  if (n_admit <= kAdmitList) {
    for (int32_t i = warp; i < n_admit; i += kTurnThreads / 32) {
      int32_t* c = a.config_pool + static_cast<int64_t>(admit[i]) * NCFG;
      for (int k = lane; k < NCFG; k += 32) c[k] = init_s[k];
    }
  } else {
    for (int32_t r = warp; r < a.rows; r += kTurnThreads / 32) {
      if (a.retired[r] == 0 || a.kind[r] != 1) continue;
      int32_t* c = a.config_pool + static_cast<int64_t>(r) * NCFG;
      for (int k = lane; k < NCFG; k += 32) c[k] = init_s[k];
    }
  }
  int32_t j = 0;
  for (int32_t r0 = 0; r0 < a.rows; r0 += kTurnThreads, ++j) {
    const int32_t r = r0 + tid;
    int32_t k = -1;
    if (r < a.rows) k = j < kRowsInRegs ? kinds[j < kRowsInRegs ? j : 0] : a.kind[r];
    const uint32_t bd = __ballot_sync(0xFFFFFFFFu, k == 0), bp = __ballot_sync(0xFFFFFFFFu, k == 1);
    if (lane == 0) {
      warp_d[warp] = __popc(bd);
      warp_p[warp] = __popc(bp);
    }
    __syncthreads();
    int32_t od = base_d, op = base_p;
    for (int i = 0; i < warp; ++i) {
      od += warp_d[i];
      op += warp_p[i];
    }
    const uint32_t below = (1u << lane) - 1u;
    if (k == 0) a.dense_rows[od + __popc(bd & below)] = r;
    if (k == 1) a.pda_rows[op + __popc(bp & below)] = r;
    __syncthreads();
    if (tid == kTurnThreads - 1) {
      base_d = od + __popc(bd);
      base_p = op + __popc(bp);
    }
    __syncthreads();
  }
  if (tid == 0) {
    a.counts[0] = base_d;
    a.counts[1] = base_p;
    *a.step = step + 1;
  }
}

// tokens_out[dense_rows[b]] = dense_tok[b] for b < counts[0], and likewise
// for the PDA list.
__global__ void gather_tokens_kernel(int32_t rows, const int64_t* __restrict__ dense_rows,
                                     const int64_t* __restrict__ pda_rows,
                                     const int32_t* __restrict__ counts,
                                     const int64_t* __restrict__ dense_tok,
                                     const int64_t* __restrict__ pda_tok,
                                     int64_t* __restrict__ tokens_out) {
  pdl_trigger();
  pdl_wait();
  const int32_t b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= rows) return;
  const int32_t nd = min(counts[0], rows), np = min(counts[1], rows);
  if (b < nd) {
    const int64_t r = dense_rows[b];
    if (r >= 0 && r < rows) tokens_out[r] = dense_tok[b];
  }
  if (b < np) {
    const int64_t r = pda_rows[b];
    if (r >= 0 && r < rows) tokens_out[r] = pda_tok[b];
  }
}

}  // namespace
}  // namespace bpd

using namespace bpd;

extern "C" bpd_status bpd_serving_turnover(
    int32_t rows, uint64_t seed, uint64_t* step_counter, float evict_prob, float p_regex,
    float p_schema, int32_t n_regex, int32_t schema_grammar, const int32_t* dense_starts,
    const int32_t* pda_init, int32_t* kind, int32_t* state_pool, int32_t* config_pool,
    uint8_t* broken, int64_t* dense_rows, int64_t* pda_rows, int32_t* counts, uint8_t* retired,
    void* stream) {
  BPD_REQUIRE(rows >= 0, "bpd_serving_turnover: bad rows");
  if (rows == 0) return BPD_OK;
  BPD_REQUIRE(step_counter && dense_starts && pda_init && kind && state_pool && config_pool &&
                  broken && dense_rows && pda_rows && counts && retired,
              "bpd_serving_turnover: null pointer");
  BPD_REQUIRE(n_regex >= 1, "bpd_serving_turnover: n_regex must be >= 1");
  BPD_REQUIRE(evict_prob >= 0.0f && evict_prob <= 1.0f && p_regex >= 0.0f && p_schema >= 0.0f &&
                  p_regex + p_schema <= 1.0f,
              "bpd_serving_turnover: probabilities out of range");
  TurnArgs a{rows,       seed,   step_counter, evict_prob, p_regex,    p_schema,
             n_regex,    schema_grammar,       dense_starts, pda_init, kind,
             state_pool, config_pool,          broken,       dense_rows, pda_rows,
             counts,     retired};
  const cudaError_t e = launch_pdl(turnover_kernel, dim3(1), dim3(kTurnThreads), 0,
                                   as_stream(stream), a);
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "turnover_kernel: %s", cudaGetErrorString(e));
  return check_launch("turnover_kernel");
}

extern "C" bpd_status bpd_serving_gather_tokens(int32_t rows, const int64_t* dense_rows,
                                                const int64_t* pda_rows, const int32_t* counts,
                                                const int64_t* dense_tok, const int64_t* pda_tok,
                                                int64_t* tokens_out, void* stream) {
  BPD_REQUIRE(rows >= 0, "bpd_serving_gather_tokens: bad rows");
  if (rows == 0) return BPD_OK;
  BPD_REQUIRE(dense_rows && pda_rows && counts && dense_tok && pda_tok && tokens_out,
              "bpd_serving_gather_tokens: null pointer");
  const cudaError_t e = launch_pdl(gather_tokens_kernel, dim3((rows + 255) / 256), dim3(256), 0,
                                   as_stream(stream), rows, dense_rows, pda_rows, counts,
                                   dense_tok, pda_tok, tokens_out);
  if (e != cudaSuccess)
    return fail(BPD_ERR_CUDA, "gather_tokens_kernel: %s", cudaGetErrorString(e));
  return check_launch("gather_tokens_kernel");
}
