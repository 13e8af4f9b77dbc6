// Row streaming shared by the dense and PDA mask kernels: mask one segment of
// a logits row against a packed allow row with 16-byte vector accesses, and
// optionally track the row's first maximal element (torch.argmax order).
//
// Per 16-byte vector: all tokens allowed -> untouched (loaded only when the
// argmax needs the values); all rejected -> one store of neg_inf, no load;
// mixed -> load, blend, store.
#pragma once

#include <climits>
#include <type_traits>

#include <cooperative_groups.h>

#include "common.cuh"

namespace bpd {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
#ifndef BPD_VPT
#define BPD_VPT 4
#endif
constexpr int kVPT = BPD_VPT;  // 16-byte vectors per lane per warp tile
constexpr unsigned kAll = 0xFFFFFFFFu;

template <typename T>
constexpr int tile_elems() {
  return 32 * kVPT * Dt<T>::kPerVec;
}

// First-maximal element of a thread's share of a row, as (key, index) with
// key = order_key(value); merged lexicographically, so the order of merging
// does not matter.
struct ArgState {
  uint32_t key = 0;       // order_key of the best value seen (0 = none yet)
  int32_t idx = INT_MAX;  // its index (the first one with that key)
};

// max() that returns NaN when either input is NaN.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Largest element of a 16-byte vector as fp32 (NaN if any element is NaN).
template <typename T>
__device__ __forceinline__ float vec_max(const uint4& v) {
  if constexpr (sizeof(typename Dt<T>::Bits) == 4) {
    return fmax_nan(fmax_nan(__uint_as_float(v.x), __uint_as_float(v.y)),
                    fmax_nan(__uint_as_float(v.z), __uint_as_float(v.w)));
  } else if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162 m = __hmax2_nan(__hmax2_nan(p[0], p[1]), __hmax2_nan(p[2], p[3]));
    const uint32_t u = *reinterpret_cast<const uint32_t*>(&m);
    return fmax_nan(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
  } else {
    const __half2* p = reinterpret_cast<const __half2*>(&v);
    const __half2 m = __hmax2_nan(__hmax2_nan(p[0], p[1]), __hmax2_nan(p[2], p[3]));
    return fmax_nan(__low2float(m), __high2float(m));
  }
}

// Fold element `idx` with value `x` into the running best (ties: lower index).
__device__ __forceinline__ void arg_elem(ArgState& st, float x, int32_t idx) {
  const uint32_t k = order_key(x);
  if (k > st.key || (k == st.key && idx < st.idx)) {
    st.key = k;
    st.idx = idx;
  }
}

// Running best VECTOR of a thread that visits its vectors in increasing index
// order: the largest vector maximum (NaN above everything, -0 == +0) and the
// first vector that reached it. Folding a vector is a few branch-free
// instructions, the same for every lane of a warp; the element inside the
// winning vector is found once, at the end (vec_arg_resolve).
struct VecArg {
  float best = 0.0f;
  int32_t vec = INT_MAX;  // element index of the winning vector (INT_MAX: none)
};

__device__ __forceinline__ void vec_arg_fold(VecArg& a, float m, int32_t e0) {
  const bool take = (a.vec == INT_MAX) | (m > a.best) | ((m != m) & (a.best == a.best));
  a.best = take ? m : a.best;
  a.vec = take ? e0 : a.vec;
}

// Merge the winning vector's first maximal element into `st`. The vector is
// read back from `row`: this thread wrote it (or left it untouched) itself.
template <typename T>
__device__ __forceinline__ void vec_arg_resolve(ArgState& st, const VecArg& a, const T* row) {
  if (a.vec == INT_MAX) return;
  const uint4 v = *reinterpret_cast<const uint4*>(row + a.vec);
  const uint32_t k = order_key(a.best);
  int32_t first = 0;
#pragma unroll
  for (int i = Dt<T>::kPerVec - 1; i >= 0; --i)
    if (order_key(Dt<T>::to_float(vec_get<T>(v, i))) == k) first = i;
  if (k > st.key || (k == st.key && a.vec + first < st.idx)) {
    st.key = k;
    st.idx = a.vec + first;
  }
}

// One element of apply_soft_: -inf where the bias is -inf (disallowed),
// otherwise logits + alpha * bias (the add skipped when alpha == 0) computed
// in fp32 and rounded once to the logits dtype.
template <typename T>
__device__ __forceinline__ typename Dt<T>::Bits soft_one(typename Dt<T>::Bits x, float bias,
                                                         float alpha) {
  if (bias == -INFINITY) return Dt<T>::from_float_dev(-INFINITY);
  if (alpha == 0.0f) return x;
  return Dt<T>::from_float_dev(fmaf(alpha, bias, Dt<T>::to_float(x)));
}

// soft_one over a 16-byte logits vector and its EPV biases.
template <typename T>
__device__ __forceinline__ uint4 soft_vec(const uint4& x, const float4* b, float alpha) {
  using Bits = typename Dt<T>::Bits;
  constexpr int EPV = Dt<T>::kPerVec;
  uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < EPV; ++i) {
    const float4& f = b[i >> 2];
    const float bi = (i & 3) == 0 ? f.x : (i & 3) == 1 ? f.y : (i & 3) == 2 ? f.z : f.w;
    const Bits y = soft_one<T>(vec_get<T>(x, i), bi, alpha);
    if constexpr (sizeof(Bits) == 4) {
      w[i] = y;
    } else {
      w[i >> 1] = (i & 1) ? ((w[i >> 1] & 0xFFFFu) | (uint32_t(y) << 16))
                          : ((w[i >> 1] & 0xFFFF0000u) | uint32_t(y));
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Shared memory of one streaming CTA: a buffer of fill values that bulk
// stores copy from, one flag byte per warp tile, then the staged allow words.
constexpr int32_t kFillBytes = 8192;

template <typename T>
__host__ __device__ constexpr int32_t stream_tiles(int32_t chunk) {
  return (chunk + tile_elems<T>() - 1) / tile_elems<T>();
}

template <typename T>
__host__ __device__ constexpr size_t stream_smem_bytes(int32_t chunk) {
  return kFillBytes + ((static_cast<size_t>(stream_tiles<T>(chunk)) + 15) & ~static_cast<size_t>(15)) +
         sizeof(uint32_t) * static_cast<size_t>((chunk + 31) / 32 + 1);
}

// Bulk (TMA engine) store of `bytes` (a multiple of 16) of fill values to a
// 16-byte aligned global address, in pieces of at most kFillBytes.
__device__ __forceinline__ void bulk_fill(void* dst, uint32_t bytes, const uint4* sfill) {
  const uint32_t src = static_cast<uint32_t>(__cvta_generic_to_shared(sfill));
  char* d = static_cast<char*>(dst);
  for (uint32_t off = 0; off < bytes; off += kFillBytes) {
    const uint32_t n = min(static_cast<uint32_t>(kFillBytes), bytes - off);
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(d + off),
                 "r"(src), "r"(n)
                 : "memory");
  }
}

// Masks [c0, c1) of `row` (c0 a multiple of the warp tile, so allow words line
// up) against allow row `brow` (nullptr = reject everything). With kArgmax the
// thread also tracks the first maximal element of the masked row (rejected
// elements count with the fill value, exactly as torch.argmax sees the row).
//
// 1. The chunk's allow words are staged into shared memory with independent
//    loads (one latency for the chunk, not one dependent L2 trip per tile).
// 2. Tiles (TILE elements) with no allowed token are flagged; thread 0 writes
//    every run of them with the bulk-copy (TMA) engine from a buffer of fill
//    values -- no per-element instructions -- and only waits for the engine
//    to have read the buffer before the CTA may exit.
// 3. The other tiles stream through registers, interleaved across warps so a
//    CTA's accesses stay within one window: all-allowed vectors are not
//    written (loaded only for the argmax), rejected vectors are stored without
//    a load, mixed ones loaded, blended and stored.
// With kArgmax a thread folds its vectors (in increasing index order) into a
// VecArg, resolved at the end; the bulk-filled runs and the scalar tail's
// fills only lower `fill_first`. All threads of the CTA must call this.
//
// With kSoft the chunk gets apply_soft_ instead of the plain mask: `lrow` is
// the row's lookahead biases (finite only where `brow` allows, so dead tiles
// and all-rejected vectors are the same -inf fill), and every live vector
// loads its logits and its biases together and is always written.
template <typename T, bool kVec, bool kArgmax, bool kSoft = false>
__device__ __forceinline__ void mask_chunk(T* __restrict__ row, int32_t c0, int32_t c1,
                                           const uint32_t* __restrict__ brow,
                                           typename Dt<T>::Bits fill, ArgState& st,
                                           uint8_t* __restrict__ smem,
                                           const float* __restrict__ lrow = nullptr,
                                           float alpha = 0.0f) {
  using Bits = typename Dt<T>::Bits;
  constexpr int EPV = Dt<T>::kPerVec;
  constexpr int TILE = tile_elems<T>();
  constexpr int WPT = TILE / 32;  // allow words per warp tile
  constexpr uint32_t FULL = (1u << EPV) - 1u;
  uint4* sfill = reinterpret_cast<uint4*>(smem);
  uint8_t* sdead = smem + kFillBytes;
  const int32_t lane = threadIdx.x & 31;
  const int32_t warp = threadIdx.x >> 5;
  int32_t fill_first = INT_MAX;  // lowest index this thread wrote `fill` to
  VecArg va;
  const uint4 fv = vec_splat<T>(fill);
  const int32_t ntiles = (kVec && c1 > c0) ? (c1 - c0) / TILE : 0;
  uint32_t* sbits = reinterpret_cast<uint32_t*>(
      smem + kFillBytes + ((static_cast<size_t>(stream_tiles<T>(c1 - c0 > 0 ? c1 - c0 : 0)) + 15) &
                           ~static_cast<size_t>(15)));
  const int32_t w0 = c0 >> 5;
  const int32_t nw = c1 > c0 ? ((c1 + 31) >> 5) - w0 : 0;
  if (brow != nullptr) {
    for (int32_t i = threadIdx.x; i < nw; i += kThreads) sbits[i] = __ldg(brow + w0 + i);
  }
  if constexpr (kVec) {
    for (int32_t i = threadIdx.x; i < kFillBytes / 16; i += kThreads) sfill[i] = fv;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  int32_t vend = c0;
  if constexpr (kVec) {
    vend = c0 + ntiles * TILE;
    for (int32_t ti = warp; ti < ntiles; ti += kWarps) {
      const uint32_t w = (brow != nullptr && lane < WPT) ? sbits[ti * WPT + lane] : 0u;
      const bool dead = !__any_sync(kAll, w != 0u);
      if (lane == 0) sdead[ti] = dead ? 1 : 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      bool issued = false;
      for (int32_t ti = 0; ti < ntiles;) {
        if (!sdead[ti]) {
          ++ti;
          continue;
        }
        int32_t te = ti + 1;
        while (te < ntiles && sdead[te]) ++te;
        bulk_fill(row + c0 + ti * TILE, static_cast<uint32_t>((te - ti) * TILE * sizeof(T)), sfill);
        fill_first = min(fill_first, c0 + ti * TILE);
        issued = true;
        ti = te;
      }
      if (issued) {
        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      }
    }
    for (int32_t ti = warp; ti < ntiles; ti += kWarps) {
      if (sdead[ti]) continue;
      const int32_t tb = c0 + ti * TILE;
      const uint32_t w = (brow != nullptr && lane < WPT) ? sbits[ti * WPT + lane] : 0u;
      uint32_t bits[kVPT];
#pragma unroll
      for (int j = 0; j < kVPT; ++j) {
        const int v = lane + 32 * j;
        const uint32_t word = __shfl_sync(kAll, w, (v * EPV) >> 5);
        bits[j] = (word >> ((v * EPV) & 31)) & FULL;
      }
      uint4* base = reinterpret_cast<uint4*>(row + tb);
      // Lanes of a warp see different bit patterns: every step below is the
      // same instruction stream for all of them (predicated loads and store,
      // branch-free blend), so a warp never runs the cases one after another.
      // Soft vectors go in groups (logits + biases in flight together).
      constexpr int G = kSoft ? (sizeof(Bits) == 4 ? 2 : 1) : kVPT;
      constexpr int NB = kSoft ? G * (EPV / 4) : 1;
#pragma unroll
      for (int g = 0; g < kVPT; g += G) {
        uint4 val[G];
        float4 bias[NB];
#pragma unroll
        for (int jj = 0; jj < G; ++jj) {
          const int j = g + jj;
          const bool need = (kArgmax || kSoft) ? (bits[j] != 0u)
                                               : (bits[j] != 0u && bits[j] != FULL);
          val[jj] = make_uint4(0u, 0u, 0u, 0u);  // not read by the blend unless loaded
          if (need) val[jj] = __ldcs(base + lane + 32 * j);
          if constexpr (kSoft) {
            const float4* lb =
                reinterpret_cast<const float4*>(lrow + tb + (lane + 32 * j) * EPV);
#pragma unroll
            for (int q = 0; q < EPV / 4; ++q) {
              bias[jj * (EPV / 4) + q] = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
              if (need) bias[jj * (EPV / 4) + q] = __ldg(lb + q);
            }
          }
        }
#pragma unroll
        for (int jj = 0; jj < G; ++jj) {
          const int j = g + jj;
          uint4 out;
          if constexpr (kSoft) {
            out = soft_vec<T>(val[jj], &bias[jj * (EPV / 4)], alpha);
          } else {
            out = vec_blend<T>(val[jj], bits[j], fill);
          }
          if (kSoft || bits[j] != FULL) __stcs(base + lane + 32 * j, out);
          if constexpr (kArgmax) vec_arg_fold(va, vec_max<T>(out), tb + (lane + 32 * j) * EPV);
        }
      }
    }
  }
  Bits* rb = reinterpret_cast<Bits*>(row);
  for (int32_t e = vend + static_cast<int32_t>(threadIdx.x); e < c1; e += kThreads) {
    const bool allowed = brow != nullptr && ((sbits[(e >> 5) - w0] >> (e & 31)) & 1u);
    if constexpr (kSoft) {
      const Bits y = soft_one<T>(rb[e], allowed ? __ldg(lrow + e) : -INFINITY, alpha);
      rb[e] = y;
      if constexpr (kArgmax) arg_elem(st, Dt<T>::to_float(y), e);
    } else if (allowed) {
      if constexpr (kArgmax) arg_elem(st, Dt<T>::to_float(rb[e]), e);
    } else {
      rb[e] = fill;
      fill_first = min(fill_first, e);
    }
  }
  if constexpr (kArgmax) {
    vec_arg_resolve<T>(st, va, row);
    if (fill_first != INT_MAX) arg_elem(st, Dt<T>::to_float(fill), fill_first);
  }
}

// ---------------------------------------------------------------------------
// Kernels built on mask_chunk, shared by the dense and the PDA paths.

// What a row masks against: its allow words (nullptr = reject everything) and,
// for the dense commit, its state and pool slot.
struct RowInfo {
  const uint32_t* brow;
  int32_t state;
  int64_t slot;
  const float* lrow = nullptr;  // soft rows: the lookahead biases of the state
};

// Rows functors say whether they carry lookahead biases (Rows::kSoft) and
// then hold the bias scale `alpha`.
template <class Rows>
__device__ __forceinline__ float rows_alpha(const Rows& r) {
  if constexpr (Rows::kSoft) {
    return r.alpha;
  } else {
    return 0.0f;
  }
}

// Dense rows: a row's state from the pool (through its slot) picks an allow
// row; DenseCommit writes the chosen token's next state (ops.py:301-306).
__device__ __forceinline__ const uint32_t* state_row(const int32_t* __restrict__ pool,
                                                     const int64_t* __restrict__ slots,
                                                     int32_t row, const uint32_t* __restrict__ bits,
                                                     int32_t wstride, int32_t S, int32_t* state,
                                                     int64_t* slot_out) {
  const int64_t slot = slots ? slots[row] : row;
  const int32_t s = pool[slot];
  *state = s;
  if (slot_out) *slot_out = slot;
  return (s >= 0 && s < S) ? bits + static_cast<int64_t>(s) * wstride : nullptr;
}

struct DenseRows {
  static constexpr bool kSoft = false;
  const int32_t* pool;
  const int64_t* slots;
  const uint32_t* bits;
  int32_t wstride;
  int32_t S;
  __device__ __forceinline__ RowInfo operator()(int32_t row) const {
    RowInfo r;
    r.brow = state_row(pool, slots, row, bits, wstride, S, &r.state, &r.slot);
    return r;
  }
};

// Dense commit of the chosen token: next = tok_next[state, token] (ops.py:301-306).
struct DenseCommit {
  int32_t* pool;
  const int32_t* tok_next;
  int32_t S;
  int32_t V;
  int64_t* token_out;
  int32_t* next_out;
  __device__ __forceinline__ void operator()(int32_t row, const RowInfo& r, int32_t tok) const {
    const int32_t s = r.state;
    const int32_t next = (s >= 0 && s < S && tok >= 0 && tok < V)
                             ? tok_next[static_cast<int64_t>(s) * V + tok]
                             : -1;
    pool[r.slot] = next;
    token_out[row] = tok;
    if (next_out) next_out[row] = next;
  }
};

// Register cap (resident CTAs per SM) and warp tiles per warp of one apply
// CTA; tuned on B200 (8 resident CTAs beat fewer CTAs with more registers).
#ifndef BPD_APPLY_MIN_BLOCKS
#define BPD_APPLY_MIN_BLOCKS 8
#endif
#ifndef BPD_APPLY_TILES_PER_WARP
#define BPD_APPLY_TILES_PER_WARP 4
#endif
#ifndef BPD_STEP_MIN_BLOCKS
#define BPD_STEP_MIN_BLOCKS 8
#endif

// Mask only: one CTA per (row, segment); the hardware block scheduler hands
// segments of cheap and expensive rows out dynamically.
template <typename T, bool kVec, class Rows>
__global__ void __launch_bounds__(kThreads, BPD_APPLY_MIN_BLOCKS)
    stream_apply_kernel(T* __restrict__ logits, int64_t row_stride, int32_t V, Rows rows,
                        typename Dt<T>::Bits fill, int32_t chunk, int32_t chunks_per_row) {
  const int32_t row = blockIdx.x / chunks_per_row;
  const int32_t c0 = (blockIdx.x - row * chunks_per_row) * chunk;
  const int32_t c1 = min(V, c0 + chunk);
  const RowInfo info = rows(row);
  extern __shared__ __align__(16) uint8_t smem[];
  ArgState st;
  mask_chunk<T, kVec, false, Rows::kSoft>(logits + row * row_stride, c0, c1, info.brow, fill, st,
                                          smem, info.lrow, rows_alpha(rows));
}

// End of a fused step: reduce every thread's first-maximal element to the
// CTA's, write it into rank 0's shared memory (distributed shared memory),
// and after one cluster barrier let rank 0 commit the row's winning token.
// All threads of every CTA of the cluster must call this.
template <class Commit>
__device__ __forceinline__ void cluster_commit(const ArgState& st, int32_t row,
                                               const RowInfo& info, const Commit& commit) {
  __shared__ uint64_t warp_best[kWarps];
  __shared__ uint64_t cluster_best[8];
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int32_t k = static_cast<int32_t>(cluster.num_blocks());
  const int32_t rank = static_cast<int32_t>(cluster.block_rank());
  const uint64_t mine = warp_max_u64(pack_arg(st.key, st.idx));
  const int32_t lane = threadIdx.x & 31;
  const int32_t warp = threadIdx.x >> 5;
  if (lane == 0) warp_best[warp] = mine;
  __syncthreads();
  if (warp == 0) {
    uint64_t q = lane < kWarps ? warp_best[lane] : 0;
    q = warp_max_u64(q);
    if (lane == 0) {
      uint64_t* dst = cluster.map_shared_rank(cluster_best, 0);
      dst[rank] = q;
    }
  }
  cluster.sync();
  if (rank == 0 && threadIdx.x == 0) {
    uint64_t best = 0;
    for (int32_t r = 0; r < k; ++r) best = cluster_best[r] > best ? cluster_best[r] : best;
    commit(row, info, unpack_idx(best));
  }
}

// Fused greedy step: a thread-block cluster of `k` CTAs owns one row; every
// CTA masks its slice and reduces its first-maximal element; the partials are
// written into rank 0's shared memory (distributed shared memory), and after
// one cluster barrier rank 0 hands the winning token to `commit`.
template <typename T, bool kVec, class Rows, class Commit>
__global__ void __launch_bounds__(kThreads, BPD_STEP_MIN_BLOCKS)
    stream_step_kernel(T* __restrict__ logits, int64_t row_stride, int32_t V, Rows rows,
                       Commit commit, typename Dt<T>::Bits fill, int32_t chunk) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int32_t k = static_cast<int32_t>(cluster.num_blocks());
  const int32_t rank = static_cast<int32_t>(cluster.block_rank());
  const int32_t row = blockIdx.x / k;
  const int32_t c0 = rank * chunk;
  const int32_t c1 = min(V, c0 + chunk);
  const RowInfo info = rows(row);
  extern __shared__ __align__(16) uint8_t smem[];
  ArgState st;
  mask_chunk<T, kVec, true, Rows::kSoft>(logits + row * row_stride, c0, c1, info.brow, fill, st,
                                         smem, info.lrow, rows_alpha(rows));
  cluster_commit(st, row, info, commit);
}

inline bool rows_aligned(const void* logits, int64_t row_stride, size_t esize) {
  return aligned16(logits) && (row_stride * static_cast<int64_t>(esize)) % 16 == 0;
}

// The vector path also needs 16-byte aligned lookahead rows (V % 4 == 0).
template <class Rows>
bool vec_ok(const void* logits, int64_t row_stride, size_t esize, int32_t V) {
  return rows_aligned(logits, row_stride, esize) && (!Rows::kSoft || V % 4 == 0);
}

template <typename T, class Rows>
bpd_status launch_stream_apply(void* logits, int64_t row_stride, int32_t batch, int32_t V,
                               const Rows& rows, float neg_inf, cudaStream_t st,
                               const char* what) {
  constexpr int TILE = tile_elems<T>();
  const int32_t chunk = TILE * kWarps * BPD_APPLY_TILES_PER_WARP;
  const int32_t chunks = (V + chunk - 1) / chunk;
  const int64_t grid = static_cast<int64_t>(batch) * chunks;
  if (grid >= 0x7FFFFFFF) return fail(BPD_ERR_INVALID, "%s: batch too large", what);
  const auto fill = Dt<T>::from_float_host(neg_inf);
  const size_t smem = stream_smem_bytes<T>(chunk);
  T* lg = static_cast<T*>(logits);
  if (vec_ok<Rows>(logits, row_stride, sizeof(T), V)) {
    stream_apply_kernel<T, true, Rows><<<static_cast<unsigned>(grid), kThreads, smem, st>>>(
        lg, row_stride, V, rows, fill, chunk, chunks);
  } else {
    stream_apply_kernel<T, false, Rows><<<static_cast<unsigned>(grid), kThreads, smem, st>>>(
        lg, row_stride, V, rows, fill, chunk, chunks);
  }
  return check_launch(what);
}

// CTAs per row of the fused step when the caller leaves it to us: aim for
// ~1.5 waves of 8 resident CTAs on each of the 148 SMs.
inline int32_t auto_ctas_per_row(int32_t batch) {
  const int32_t want = (148 * 12 + batch - 1) / batch;
  int32_t k = 1;
  while (k < want && k < 8) k <<= 1;
  return k;
}

template <typename T, class Rows, class Commit>
bpd_status launch_stream_step(void* logits, int64_t row_stride, int32_t batch, int32_t V,
                              const Rows& rows, const Commit& commit, float neg_inf, int32_t k,
                              cudaStream_t st, const char* what) {
  constexpr int TILE = tile_elems<T>();
  const int32_t per = (V + k - 1) / k;
  const int32_t chunk = ((per + TILE - 1) / TILE) * TILE;
  const int64_t grid = static_cast<int64_t>(batch) * k;
  if (grid >= 0x7FFFFFFF) return fail(BPD_ERR_INVALID, "%s: batch too large", what);
  const auto fill = Dt<T>::from_float_host(neg_inf);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = stream_smem_bytes<T>(chunk);
  if (cfg.dynamicSmemBytes > 48 * 1024)
    return fail(BPD_ERR_INVALID, "%s: vocab too large for %d CTAs per row", what, k);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(k);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  T* lg = static_cast<T*>(logits);
  cudaError_t e;
  if (vec_ok<Rows>(logits, row_stride, sizeof(T), V)) {
    e = cudaLaunchKernelEx(&cfg, stream_step_kernel<T, true, Rows, Commit>, lg, row_stride, V,
                           rows, commit, fill, chunk);
  } else {
    e = cudaLaunchKernelEx(&cfg, stream_step_kernel<T, false, Rows, Commit>, lg, row_stride, V,
                           rows, commit, fill, chunk);
  }
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

}  // namespace bpd
