// Row streaming shared by the dense and PDA mask kernels: mask one segment of
// a logits row against a packed allow row with 16-byte vector accesses, and
// optionally track the row's first maximal element (torch.argmax order).
//
// Per 16-byte vector: all tokens allowed -> untouched (loaded only when the
// argmax needs the values); all rejected -> one store of neg_inf, no load;
// mixed -> load, blend, store.
#pragma once

#include <algorithm>
#include <climits>
#include <type_traits>

#include "common.cuh"

namespace bpd {

#ifndef BPD_THREADS
#define BPD_THREADS 256
#endif
constexpr int kThreads = BPD_THREADS;
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

// Merge the winning vector's first maximal element into `st`; `v` is that
// vector's value (read back, or computed again, by the thread that folded it).
template <typename T>
__device__ __forceinline__ void vec_arg_resolve(ArgState& st, const VecArg& a, const uint4& v) {
  if (a.vec == INT_MAX) return;
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

// Shared memory of a streaming CTA: kFillBytes of the fill value, the source
// of the bulk (TMA engine) stores that write fully rejected tiles.
constexpr int32_t kFillBytes = 8192;

// Fill the buffer and make it visible to the bulk-copy engine.
template <typename T>
__device__ __forceinline__ void fill_init(uint8_t* smem, typename Dt<T>::Bits fill) {
  uint4* sfill = reinterpret_cast<uint4*>(smem);
  const uint4 fv = vec_splat<T>(fill);
  for (int32_t i = threadIdx.x; i < kFillBytes / 16; i += kThreads) sfill[i] = fv;
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk (TMA engine) store of `bytes` (a multiple of 16) of fill values to a
// 16-byte aligned global address, in pieces of at most kFillBytes. The lines
// are marked evict-first in L2 (nothing rereads them in the step; the allow
// words and tables that are reused stay cached): -1 % on the dense step and
// -1.5 % on the soft step over a generation.
__device__ __forceinline__ void bulk_fill(void* dst, uint32_t bytes, const uint4* sfill) {
  const uint32_t src = static_cast<uint32_t>(__cvta_generic_to_shared(sfill));
  char* d = static_cast<char*>(dst);
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  for (uint32_t off = 0; off < bytes; off += kFillBytes) {
    const uint32_t n = min(static_cast<uint32_t>(kFillBytes), bytes - off);
    asm volatile(
        "cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;" ::"l"(
            d + off),
        "r"(src), "r"(n), "l"(policy)
        : "memory");
  }
}

// A read-only 16-byte load kept in L2 with evict-last priority: the soft
// step's lookahead rows, shared by every row in the same state, stay cached
// while the logits stream past them (-1.7 % on the soft step over a
// generation).
__device__ __forceinline__ float4 ldg_keep(const float4* p, uint64_t policy) {
  float4 v;
  asm volatile("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p), "l"(policy));
  return v;
}

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

// Warp tiles whose allow words a warp loads at once.
constexpr int kGroupTiles = 4;

// The 16-byte vector of working type T at element e0 of a source row of type
// S: the same bits when S == T, else (T = float) EPV elements of S widened.
template <typename T, typename S>
__device__ __forceinline__ uint4 load_src(const S* __restrict__ srow, int32_t e0) {
  if constexpr (std::is_same_v<S, T>) {
    return __ldcs(reinterpret_cast<const uint4*>(srow + e0));
  } else {
    static_assert(std::is_same_v<T, float> && sizeof(S) == 2, "fp32 from 16-bit sources");
    const uint2 h = __ldcs(reinterpret_cast<const uint2*>(srow + e0));
    if constexpr (std::is_same_v<S, __nv_bfloat16>) {
      return make_uint4(h.x << 16, h.x & 0xFFFF0000u, h.y << 16, h.y & 0xFFFF0000u);
    } else {
      return make_uint4(__float_as_uint(__half2float(__ushort_as_half(h.x & 0xFFFFu))),
                        __float_as_uint(__half2float(__ushort_as_half(h.x >> 16))),
                        __float_as_uint(__half2float(__ushort_as_half(h.y & 0xFFFFu))),
                        __float_as_uint(__half2float(__ushort_as_half(h.y >> 16))));
    }
  }
}

// Element e of a source row as working-type bits.
template <typename T, typename S>
__device__ __forceinline__ typename Dt<T>::Bits load_src_one(const S* srow, int32_t e) {
  if constexpr (std::is_same_v<S, T>) {
    return reinterpret_cast<const typename Dt<T>::Bits*>(srow)[e];
  } else {
    const uint16_t b = reinterpret_cast<const uint16_t*>(srow)[e];
    return __float_as_uint(std::is_same_v<S, __nv_bfloat16>
                               ? __uint_as_float(uint32_t(b) << 16)
                               : __half2float(__ushort_as_half(b)));
  }
}

// Allow bits of vector j of lane `lane` in a warp tile whose allow word for
// this lane is `w` (one 32-bit word per lane, spread by shuffles).
template <typename T>
__device__ __forceinline__ uint32_t tile_bits(uint32_t w, int32_t lane, int j) {
  constexpr int EPV = Dt<T>::kPerVec;
  constexpr uint32_t FULL = (1u << EPV) - 1u;
  const int v = lane + 32 * j;
  const uint32_t word = __shfl_sync(kAll, w, (v * EPV) >> 5);
  return (word >> ((v * EPV) & 31)) & FULL;
}

#ifndef BPD_PIPELINE
#define BPD_PIPELINE 1
#endif
// fp32 rows: 0 = bulk-fill only a wholly dead group of tiles, 1 = every run
// of dead tiles (as 16-bit rows do)
#ifndef BPD_F32_RUN_BULK
#define BPD_F32_RUN_BULK 0
#endif

// Head of one group of kGroupTiles warp tiles, tiles g0.. of the span
// [e0, e0 + ntiles * TILE): every lane loads its allow word of each tile into
// w (independent loads, one latency for the group), one vote per tile finds
// the tiles with no allowed token, and lane 0 writes each run of them with
// the bulk-copy engine from the fill buffer (`issued` tells the caller to
// wait for the engine before the warp exits). fp32 rows bulk-fill only a
// wholly dead group; their dead tiles among live ones take plain stores with
// the live tiles (-4 % on the PDA step, neutral on the soft step; 16-bit rows
// keep every dead tile on the bulk engine, which is faster there). Returns
// the mask of the group's tiles left for the vector path.
template <typename T>
__device__ __forceinline__ uint32_t group_head(T* row, int32_t e0, int32_t g0, int32_t ntiles,
                                               const uint32_t* __restrict__ brow,
                                               const uint4* sfill, uint32_t (&w)[kGroupTiles],
                                               int32_t lane, int32_t& fill_first,
                                               bool& issued) {
  constexpr int TILE = tile_elems<T>();
  constexpr int WPT = TILE / 32;  // allow words per warp tile
#pragma unroll
  for (int t = 0; t < kGroupTiles; ++t) {
    w[t] = 0u;
    if (brow != nullptr && g0 + t < ntiles && lane < WPT)
      w[t] = __ldg(brow + ((e0 + (g0 + t) * TILE) >> 5) + lane);
  }
  uint32_t live = 0u;
#pragma unroll
  for (int t = 0; t < kGroupTiles; ++t) live |= (__any_sync(kAll, w[t] != 0u) ? 1u : 0u) << t;
  const int32_t ng = min(kGroupTiles, ntiles - g0);
  uint32_t dead = ((1u << ng) - 1u) & ~live;
  if constexpr (sizeof(typename Dt<T>::Bits) == 4 && !BPD_F32_RUN_BULK) {
    if (dead != (1u << ng) - 1u) {
      live |= dead;
      dead = 0u;
    }
  }
  if (dead != 0u && lane == 0) {
    fill_first = min(fill_first, e0 + (g0 + __ffs(dead) - 1) * TILE);
    uint32_t d = row != nullptr ? dead : 0u;
    while (d != 0u) {
      const int t0 = __ffs(d) - 1;
      const int run = __ffs(~(d >> t0)) - 1;
      bulk_fill(row + e0 + (g0 + t0) * TILE,
                static_cast<uint32_t>(run * TILE * static_cast<int32_t>(sizeof(T))), sfill);
      d &= ~(((1u << run) - 1u) << t0);
    }
    issued = issued || row != nullptr;
  }
  return live;
}

// One warp masks [e0, e1) of `row` (e0 a multiple of the warp tile, so allow
// words line up) against allow row `brow` (nullptr = reject everything); no
// barrier, no shared state with the CTA's other warps except the read-only
// fill buffer. With kArgmax each lane also tracks the first maximal element
// of its share of the masked row (rejected elements count with the fill
// value, as torch.argmax sees the row).
//
// Per group of kGroupTiles tiles (TILE elements each):
// 1. every lane loads its allow word of each tile (independent loads, one
//    latency for the group) and one vote per tile finds the tiles with no
//    allowed token;
// 2. lane 0 writes each run of such tiles with the bulk-copy engine from the
//    fill buffer -- no per-element instructions, nothing waited for until the
//    warp exits (`issued` tells the caller to wait then);
// 3. the other tiles stream through registers with one instruction stream
//    for all lanes whatever their bit pattern: predicated loads and stores,
//    branch-free blend. All-allowed vectors are not written (loaded only for
//    the argmax), rejected ones stored without a load, mixed ones loaded,
//    blended and stored.
// A lane visits its vectors in increasing index order and folds them into a
// VecArg, resolved at the end; bulk-filled runs and the scalar tail's fills
// only lower `fill_first`.
//
// With kSoft the span gets apply_soft_ instead of the plain mask: `lrow` is
// the row's lookahead biases (finite only where `brow` allows, so dead tiles
// and all-rejected vectors are the same -inf fill), and a live vector loads
// its logits and its biases together and is always written.
//
// The warp's tiles are the contiguous span [e0, e0 + nt * TILE) (its dead
// tiles merge into runs), then it handles the scalar elements [s0, s1) one
// per lane.
//
// Source and destination: the values come from `srow` (type S) and the
// result goes to `row` (working type T). In place (kInPlace: the same row)
// all-allowed vectors are not written; otherwise every vector of `row` is,
// and `row` may be nullptr: nothing is written (only the argmax is wanted).
template <typename T, typename S, bool kInPlace, bool kVec, bool kArgmax, bool kSoft>
__device__ __forceinline__ void warp_span(T* __restrict__ row, const S* __restrict__ srow,
                                          int32_t e0, int32_t nt, int32_t s0, int32_t s1,
                                          const uint32_t* __restrict__ brow,
                                          typename Dt<T>::Bits fill, const uint4* sfill,
                                          const float* __restrict__ lrow, float alpha,
                                          ArgState& st, bool& issued) {
  using Bits = typename Dt<T>::Bits;
  constexpr int EPV = Dt<T>::kPerVec;
  constexpr int TILE = tile_elems<T>();
  constexpr uint32_t FULL = (1u << EPV) - 1u;
  const int32_t lane = threadIdx.x & 31;
  int32_t fill_first = INT_MAX;  // lowest index this lane wrote `fill` to
  VecArg va;
  if constexpr (kVec) {
    const int32_t ntiles = nt;
    for (int32_t g0 = 0; g0 < ntiles; g0 += kGroupTiles) {
      uint32_t w[kGroupTiles];
      const uint32_t live = group_head<T>(row, e0, g0, ntiles, brow, sfill, w, lane, fill_first,
                                          issued);
      if constexpr (!kSoft && BPD_PIPELINE) {
        // Software-pipelined live tiles: while tile t is blended, stored and
        // (with the argmax) folded vector by vector, the loads of tile t + 1
        // (when live) are issued into the registers each vector frees, so
        // this tile's work overlaps the next tile's memory latency.
        uint4 val[kVPT];
        bool loaded = false;  // val holds the current tile (warp-uniform)
#pragma unroll
        for (int t = 0; t < kGroupTiles; ++t) {
          if (((live >> t) & 1u) == 0u) {
            loaded = false;
            continue;
          }
          const int32_t tb = e0 + (g0 + t) * TILE;
          if (!loaded) {
#pragma unroll
            for (int j = 0; j < kVPT; ++j) {
              const uint32_t b = tile_bits<T>(w[t], lane, j);
              const bool need = (kArgmax || !kInPlace) ? (b != 0u) : (b != 0u && b != FULL);
              val[j] = make_uint4(0u, 0u, 0u, 0u);
              if (need) val[j] = load_src<T, S>(srow, tb + (lane + 32 * j) * EPV);
            }
          }
          const bool next = t + 1 < kGroupTiles && ((live >> (t + 1)) & 1u) != 0u;
          const int32_t nb = tb + TILE;
          uint4* base = reinterpret_cast<uint4*>(row + tb);
#pragma unroll
          for (int j = 0; j < kVPT; ++j) {
            const uint32_t b = tile_bits<T>(w[t], lane, j);
            const uint4 out = vec_blend<T>(val[j], b, fill);
            if (row != nullptr && (!kInPlace || b != FULL)) __stcs(base + lane + 32 * j, out);
            if (next) {
              const uint32_t bn = tile_bits<T>(w[t + 1 < kGroupTiles ? t + 1 : t], lane, j);
              const bool need = (kArgmax || !kInPlace) ? (bn != 0u) : (bn != 0u && bn != FULL);
              val[j] = make_uint4(0u, 0u, 0u, 0u);
              if (need) val[j] = load_src<T, S>(srow, nb + (lane + 32 * j) * EPV);
            }
            if constexpr (kArgmax) vec_arg_fold(va, vec_max<T>(out), tb + (lane + 32 * j) * EPV);
          }
          loaded = next;
        }
      } else {
      uint64_t keep = 0;
      if constexpr (kSoft) keep = l2_evict_last_policy();
#pragma unroll
      for (int t = 0; t < kGroupTiles; ++t) {
        if (((live >> t) & 1u) == 0u) continue;  // the same for the whole warp
        const int32_t tb = e0 + (g0 + t) * TILE;
        uint32_t bits[kVPT];
#pragma unroll
        for (int j = 0; j < kVPT; ++j) {
          const int v = lane + 32 * j;
          const uint32_t word = __shfl_sync(kAll, w[t], (v * EPV) >> 5);
          bits[j] = (word >> ((v * EPV) & 31)) & FULL;
        }
        uint4* base = reinterpret_cast<uint4*>(row + tb);
        // soft vectors go in groups (logits + biases in flight together)
        constexpr int G = kSoft ? (sizeof(Bits) == 4 ? 2 : 1) : kVPT;
        constexpr int NB = kSoft ? G * (EPV / 4) : 1;
#pragma unroll
        for (int g = 0; g < kVPT; g += G) {
          uint4 val[G];
          float4 bias[NB];
#pragma unroll
          for (int jj = 0; jj < G; ++jj) {
            const int j = g + jj;
            const bool need = (kArgmax || kSoft || !kInPlace)
                                  ? (bits[j] != 0u)
                                  : (bits[j] != 0u && bits[j] != FULL);
            val[jj] = make_uint4(0u, 0u, 0u, 0u);  // not read by the blend unless loaded
            if (need) val[jj] = load_src<T, S>(srow, tb + (lane + 32 * j) * EPV);
            if constexpr (kSoft) {
              const float4* lb =
                  reinterpret_cast<const float4*>(lrow + tb + (lane + 32 * j) * EPV);
#pragma unroll
              for (int q = 0; q < EPV / 4; ++q) {
                bias[jj * (EPV / 4) + q] =
                    make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
                if (need) bias[jj * (EPV / 4) + q] = ldg_keep(lb + q, keep);
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
            if (row != nullptr && (kSoft || !kInPlace || bits[j] != FULL))
              __stcs(base + lane + 32 * j, out);
            if constexpr (kArgmax)
              vec_arg_fold(va, vec_max<T>(out), tb + (lane + 32 * j) * EPV);
          }
        }
      }
      }
    }
    if (issued) asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
  Bits* rb = reinterpret_cast<Bits*>(row);
  for (int32_t e = s0 + lane; e < s1; e += 32) {
    const bool allowed = brow != nullptr && ((__ldg(brow + (e >> 5)) >> (e & 31)) & 1u);
    if constexpr (kSoft) {
      const Bits y =
          soft_one<T>(load_src_one<T, S>(srow, e), allowed ? __ldg(lrow + e) : -INFINITY, alpha);
      if (rb != nullptr) rb[e] = y;
      if constexpr (kArgmax) arg_elem(st, Dt<T>::to_float(y), e);
    } else if (allowed) {
      const Bits x = load_src_one<T, S>(srow, e);
      if (!kInPlace && rb != nullptr) rb[e] = x;
      if constexpr (kArgmax) arg_elem(st, Dt<T>::to_float(x), e);
    } else {
      if (rb != nullptr) rb[e] = fill;
      fill_first = min(fill_first, e);
    }
  }
  if constexpr (kArgmax) {
    if (va.vec != INT_MAX) {
      // the winning vector: read back what this lane stored, or compute it
      // again from the source when nothing was stored
      uint4 v;
      if (row != nullptr) {
        v = *reinterpret_cast<const uint4*>(row + va.vec);
      } else {
        const uint32_t wd = brow != nullptr ? __ldg(brow + (va.vec >> 5)) : 0u;
        const uint32_t bits = (wd >> (va.vec & 31)) & FULL;
        const uint4 x = load_src<T, S>(srow, va.vec);
        if constexpr (kSoft) {
          float4 b[EPV / 4];
#pragma unroll
          for (int q = 0; q < EPV / 4; ++q)
            b[q] = __ldg(reinterpret_cast<const float4*>(lrow + va.vec) + q);
          v = soft_vec<T>(x, b, alpha);
        } else {
          v = vec_blend<T>(x, bits, fill);
        }
      }
      vec_arg_resolve<T>(st, va, v);
    }
    if (fill_first != INT_MAX) arg_elem(st, Dt<T>::to_float(fill), fill_first);
  }
}

#ifndef BPD_STAGED
#define BPD_STAGED 1
#endif

// Shared memory each warp of a staged kernel holds for its group of tiles.
constexpr int32_t kStageWarpBytes = kGroupTiles * 32 * kVPT * 16;
constexpr int32_t kStageBytes = kWarps * kStageWarpBytes;

// Per-thread asynchronous 16-byte copy global -> shared (L1 bypassed), and
// its group bookkeeping: the copies a thread issued before a commit form one
// group; wait_group<N> returns once at most N of the thread's groups are
// still in flight.
__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* gptr) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr), "l"(gptr) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// wait_group with a count known after unrolling (the switch folds away).
__device__ __forceinline__ void cp_async_wait_n(int n) {
  static_assert(kGroupTiles <= 4, "cp_async_wait_n covers counts 0..3");
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    default: cp_async_wait<3>(); break;
  }
}

// warp_span for an in-place mask of 16-byte aligned rows (no soft bias), with
// the live tiles of a group staged through shared memory instead of
// registers: after the group head, every lane issues one asynchronous
// 16-byte copy per vector that holds an allowed token (per vector the
// argmax or the blend needs, as in warp_span) for ALL the group's live tiles
// at once -- one commit group per tile -- so a warp keeps up to kGroupTiles
// tiles (8 KB) of loads in flight without holding them in registers. It
// then takes the tiles in order as their groups land: each lane reads back
// only the vectors it copied itself (its own cp.async.wait_group orders
// them), blends, stores the changed vectors and folds the argmax, exactly
// as warp_span does. A stage slot is refilled only by the next group, whose
// copies are issued after this group's values were consumed by stores and
// folds that depend on them. `stage` is this warp's kStageWarpBytes.
template <typename T, bool kArgmax>
__device__ __forceinline__ void warp_span_staged(T* __restrict__ row, int32_t e0, int32_t nt,
                                                 int32_t s0, int32_t s1,
                                                 const uint32_t* __restrict__ brow,
                                                 typename Dt<T>::Bits fill, const uint4* sfill,
                                                 uint4* stage, ArgState& st, bool& issued) {
  using Bits = typename Dt<T>::Bits;
  constexpr int EPV = Dt<T>::kPerVec;
  constexpr int TILE = tile_elems<T>();
  constexpr int VPT = 32 * kVPT;  // 16-byte vectors per warp tile
  constexpr uint32_t FULL = (1u << EPV) - 1u;
  static_assert(EPV * kVPT <= 32, "a tile's bits of one lane fit one word");
  const int32_t lane = threadIdx.x & 31;
  int32_t fill_first = INT_MAX;
  VecArg va;
  const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(stage));
  for (int32_t g0 = 0; g0 < nt; g0 += kGroupTiles) {
    uint32_t w[kGroupTiles];
    const uint32_t live = group_head<T>(row, e0, g0, nt, brow, sfill, w, lane, fill_first,
                                        issued);
    // this lane's bits of its kVPT vectors of each tile, packed EPV bits each
    uint32_t lb[kGroupTiles];
#pragma unroll
    for (int t = 0; t < kGroupTiles; ++t) {
      lb[t] = 0u;
#pragma unroll
      for (int j = 0; j < kVPT; ++j) lb[t] |= tile_bits<T>(w[t], lane, j) << (j * EPV);
    }
#pragma unroll
    for (int t = 0; t < kGroupTiles; ++t) {
      if ((live >> t) & 1u) {
        const T* tp = row + e0 + (g0 + t) * TILE;
#pragma unroll
        for (int j = 0; j < kVPT; ++j) {
          const uint32_t b = (lb[t] >> (j * EPV)) & FULL;
          const bool need = kArgmax ? (b != 0u) : (b != 0u && b != FULL);
          const int v = lane + 32 * j;
          if (need) cp_async16(sbase + static_cast<uint32_t>((t * VPT + v) * 16), tp + v * EPV);
        }
      }
      cp_async_commit();
    }
#pragma unroll
    for (int t = 0; t < kGroupTiles; ++t) {
      cp_async_wait_n(kGroupTiles - 1 - t);
      if (((live >> t) & 1u) == 0u) continue;
      const int32_t tb = e0 + (g0 + t) * TILE;
      uint4* base = reinterpret_cast<uint4*>(row + tb);
#pragma unroll
      for (int j = 0; j < kVPT; ++j) {
        const uint32_t b = (lb[t] >> (j * EPV)) & FULL;
        const bool need = kArgmax ? (b != 0u) : (b != 0u && b != FULL);
        const int v = lane + 32 * j;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (need) val = stage[t * VPT + v];
        const uint4 out = vec_blend<T>(val, b, fill);
        if (b != FULL) __stcs(base + v, out);
        if constexpr (kArgmax) vec_arg_fold(va, vec_max<T>(out), tb + v * EPV);
      }
    }
  }
  if (issued) asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  Bits* rb = reinterpret_cast<Bits*>(row);
  for (int32_t e = s0 + lane; e < s1; e += 32) {
    const bool allowed = brow != nullptr && ((__ldg(brow + (e >> 5)) >> (e & 31)) & 1u);
    if (allowed) {
      if constexpr (kArgmax) arg_elem(st, Dt<T>::to_float(rb[e]), e);
    } else {
      rb[e] = fill;
      fill_first = min(fill_first, e);
    }
  }
  if constexpr (kArgmax) {
    if (va.vec != INT_MAX) {
      // the winning vector, read back from the row (every lane's own stores
      // and the untouched all-allowed vectors)
      vec_arg_resolve<T>(st, va, *reinterpret_cast<const uint4*>(row + va.vec));
    }
    if (fill_first != INT_MAX) arg_elem(st, Dt<T>::to_float(fill), fill_first);
  }
}

// ---------------------------------------------------------------------------
// Kernels built on warp_span, shared by the dense, soft and PDA paths. A CTA
// owns `chunk` elements of one row (kWarps equal spans, one per warp); the
// hardware block scheduler hands CTAs of cheap and expensive rows out
// dynamically.

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

// A Rows functor gives a row's RowInfo in two steps, so that a persistent
// warp can issue the loads for its next row while it streams the current
// one: pre(row) only loads (its results are consumed later), info(row, pre)
// does the arithmetic. operator()(row) is both at once.
struct StatePre {
  int64_t slot;
  int32_t state;
};

__device__ __forceinline__ StatePre state_pre(const int32_t* __restrict__ pool,
                                              const int64_t* __restrict__ slots, int32_t row) {
  StatePre p;
  p.slot = slots ? slots[row] : row;
  p.state = pool[p.slot];
  return p;
}

struct DenseRows {
  static constexpr bool kSoft = false;
  using Pre = StatePre;
  const int32_t* pool;
  const int64_t* slots;
  const uint32_t* bits;
  int32_t wstride;
  int32_t S;
  __device__ __forceinline__ Pre pre(int32_t row) const { return state_pre(pool, slots, row); }
  __device__ __forceinline__ RowInfo info(int32_t, const Pre& p) const {
    RowInfo r;
    r.state = p.state;
    r.slot = p.slot;
    r.brow = (p.state >= 0 && p.state < S) ? bits + static_cast<int64_t>(p.state) * wstride
                                           : nullptr;
    return r;
  }
  __device__ __forceinline__ RowInfo operator()(int32_t row) const {
    RowInfo r;
    r.brow = state_row(pool, slots, row, bits, wstride, S, &r.state, &r.slot);
    return r;
  }
};

// Dense commit of the chosen token: next = tok_next[state, token] (ops.py:301-306).
// A Commit is called by all 32 lanes of the one warp that finishes a row,
// with kSmemBytes of shared memory of its own.
struct DenseCommit {
  static constexpr int kSmemBytes = 0;
  int32_t* pool;
  const int32_t* tok_next;
  int32_t S;
  int32_t V;
  int64_t* token_out;
  int32_t* next_out;
  __device__ __forceinline__ void operator()(int32_t row, const RowInfo& r, int32_t tok,
                                             uint8_t*) const {
    if ((threadIdx.x & 31) != 0) return;
    const int32_t s = r.state;
    const int32_t next = (s >= 0 && s < S && tok >= 0 && tok < V)
                             ? tok_next[static_cast<int64_t>(s) * V + tok]
                             : -1;
    pool[r.slot] = next;
    token_out[row] = tok;
    if (next_out) next_out[row] = next;
  }
};

// Register cap (resident CTAs per SM) and warp tiles per warp of a CTA,
// tuned on B200: every streaming kernel runs at 48 registers (5 CTAs of 256
// threads per SM) rather than 32 (8 CTAs). Against 8 CTAs at 32 registers:
// fused dense step -11 % in late steps (the pipelined tile loop), mask-only
// launches -5 % over a config-2 generation (pipelined too; +11 % on the first
// step alone), fused soft step -7 % over a generation, soft apply -7 %.
#ifndef BPD_APPLY_MIN_BLOCKS
#define BPD_APPLY_MIN_BLOCKS 5
#endif
#ifndef BPD_STEP_MIN_BLOCKS
#define BPD_STEP_MIN_BLOCKS 5
#endif
#ifndef BPD_SOFT_STEP_MIN_BLOCKS
#define BPD_SOFT_STEP_MIN_BLOCKS 5
#endif
#ifndef BPD_TILES_PER_WARP
#define BPD_TILES_PER_WARP 4
#endif
// Resident CTAs per SM of the staged kernels (shared memory bound: the fill
// buffer and 64 KB of stage per CTA).
#ifndef BPD_STAGED_MIN_BLOCKS
#define BPD_STAGED_MIN_BLOCKS 3
#endif

// Whether a streaming kernel instantiation stages its live tiles through
// shared memory (warp_span_staged): the in-place mask without soft bias.
template <bool kVec, bool kInPlace, class Rows>
constexpr bool staged_path() {
  return BPD_STAGED != 0 && kVec && kInPlace && !Rows::kSoft;
}

// Dynamic shared memory of a streaming CTA: the fill buffer, the stage of a
// staged kernel, then the commit's own bytes.
template <bool kStaged>
constexpr size_t stream_smem_bytes(size_t commit_bytes) {
  // staged: the committing warp's stage slice holds the commit's bytes
  return static_cast<size_t>(kFillBytes) +
         (kStaged ? static_cast<size_t>(kStageBytes) : commit_bytes);
}

// Chunk of one CTA: `chunks_per_row` CTAs per row when the caller asks for
// it, else BPD_TILES_PER_WARP warp tiles per warp. Always a multiple of
// kWarps warp tiles, so every warp span starts on a tile.
//
// With `batch` given, small batches are cut finer (down to one warp tile per
// warp) until the grid has about one CTA per SM, so a step over a handful of
// rows is not a few CTAs working through their tiles one after another
// (B = 1, V = 128,256: 13.9 -> 11.9 us per step replayed from a graph).
template <typename T>
inline int32_t stream_chunk(int32_t V, int32_t chunks_per_row, int32_t batch = 0) {
  constexpr int32_t UNIT = tile_elems<T>() * kWarps;
  if (chunks_per_row <= 0) {
    int32_t tpw = BPD_TILES_PER_WARP;
    const int64_t want = static_cast<int64_t>(sm_count());
    while (tpw > 1 && batch > 0 &&
           static_cast<int64_t>(batch) * ((V + UNIT * tpw - 1) / (UNIT * tpw)) < want)
      tpw /= 2;
    return UNIT * tpw;
  }
  const int32_t per = (V + chunks_per_row - 1) / chunks_per_row;
  return ((per + UNIT - 1) / UNIT) * UNIT;
}

// This warp's share of the CTA chunk [c0, c1): with the vector path, a
// contiguous run of the chunk's full tiles (so rejected tiles merge into
// larger bulk stores: -3 % on the dense bf16 step, -4 % on the fp32 soft step
// against tiles interleaved across warps) and, for the last warp, the ragged
// end; without the vector path a contiguous element range.
struct WarpShare {
  int32_t e0, nt, s0, s1;
};

template <typename T, bool kVec>
__device__ __forceinline__ WarpShare warp_share(int32_t c0, int32_t c1) {
  constexpr int32_t TILE = tile_elems<T>();
  const int32_t w = static_cast<int32_t>(threadIdx.x >> 5);
  WarpShare r;
  if constexpr (kVec) {
    const int32_t ntc = c1 > c0 ? (c1 - c0) / TILE : 0;
    const int32_t per = (ntc + kWarps - 1) / kWarps;
    r.e0 = c0 + w * per * TILE;
    r.nt = max(0, min(per, ntc - w * per));
    r.s0 = c0 + ntc * TILE;
    r.s1 = w == kWarps - 1 ? max(r.s0, c1) : r.s0;
  } else {
    const int32_t span = (c1 - c0 + kWarps - 1) / kWarps;
    r.e0 = c0;
    r.nt = 0;
    r.s0 = min(c1, c0 + w * span);
    r.s1 = min(c1, r.s0 + span);
  }
  return r;
}

// Mask only: one CTA per (row, chunk).
template <typename T, bool kVec, class Rows>
__global__ void __launch_bounds__(kThreads, staged_path<kVec, true, Rows>()
                                                ? BPD_STAGED_MIN_BLOCKS
                                                : BPD_APPLY_MIN_BLOCKS)
    stream_apply_kernel(T* __restrict__ logits, int64_t row_stride, int32_t V, Rows rows,
                        typename Dt<T>::Bits fill, int32_t chunk, int32_t chunks_per_row) {
  extern __shared__ __align__(16) uint8_t smem[];
  if constexpr (kVec) {
    fill_init<T>(smem, fill);
    __syncthreads();
  }
  const int32_t row = blockIdx.x / chunks_per_row;
  const int32_t c0 = (blockIdx.x - row * chunks_per_row) * chunk;
  const WarpShare ws = warp_share<T, kVec>(c0, min(V, c0 + chunk));
  const RowInfo info = rows(row);
  ArgState st;
  bool issued = false;
  T* rowp = logits + row * row_stride;
  if constexpr (staged_path<kVec, true, Rows>()) {
    uint4* stage = reinterpret_cast<uint4*>(smem + kFillBytes +
                                            (threadIdx.x >> 5) * kStageWarpBytes);
    warp_span_staged<T, false>(rowp, ws.e0, ws.nt, ws.s0, ws.s1, info.brow, fill,
                               reinterpret_cast<const uint4*>(smem), stage, st, issued);
  } else {
    warp_span<T, T, true, kVec, false, Rows::kSoft>(rowp, rowp, ws.e0, ws.nt, ws.s0,
                                                    ws.s1, info.brow, fill,
                                                    reinterpret_cast<const uint4*>(smem),
                                                    info.lrow, rows_alpha(rows), st, issued);
  }
  if (issued) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Device scratch of the fused step: per row the best packed (key, ~index) so
// far and the number of pieces done, and the persistent kernel's work queue
// (next item, warps finished). It must be zero before a launch; every launch
// that runs to completion leaves it zero again (the row's last piece clears
// the row's words, the last warp out clears the queue).
struct StepScratch {
  unsigned long long* best;  // [batch]
  uint32_t* done;            // [batch]
  uint32_t* queue;           // [2]
};

constexpr size_t step_scratch_bytes(int32_t batch) {
  return align256(sizeof(unsigned long long) * static_cast<size_t>(batch)) +
         align256(sizeof(uint32_t) * static_cast<size_t>(batch)) + 256;
}

inline StepScratch step_scratch_view(void* base, int32_t batch) {
  char* p = static_cast<char*>(base);
  StepScratch s;
  s.best = reinterpret_cast<unsigned long long*>(p);
  p += align256(sizeof(unsigned long long) * static_cast<size_t>(batch));
  s.done = reinterpret_cast<uint32_t*>(p);
  p += align256(sizeof(uint32_t) * static_cast<size_t>(batch));
  s.queue = reinterpret_cast<uint32_t*>(p);
  return s;
}

// Fused greedy step: one CTA per (row, chunk), one span per warp. Each warp
// masks its span and reduces its first-maximal element; the partials of a
// row meet in one 64-bit atomicMax of the packed (key, ~index), and the warp
// that finishes the row last (an acquire-release atomic count -- the
// last-block pattern, nothing ever waits) hands the winner to `commit`
// (all its lanes, with Commit::kSmemBytes of shared memory).
//
// In place (S == T, kInPlace) the row is `logits` row `row`. Otherwise the
// values come from source row `src_rows[row]` (row `row` when nullptr) of
// `src` (type S) and the result goes to row `row` of `logits` (working type
// T), or nowhere when `logits` is nullptr.
template <typename T, typename S, bool kInPlace, bool kVec, class Rows, class Commit>
__global__ void __launch_bounds__(kThreads,
                                  Rows::kSoft ? BPD_SOFT_STEP_MIN_BLOCKS
                                  : staged_path<kVec, kInPlace, Rows>() ? BPD_STAGED_MIN_BLOCKS
                                                                         : BPD_STEP_MIN_BLOCKS)
    stream_step_kernel(T* __restrict__ logits, int64_t row_stride, const S* __restrict__ src,
                       int64_t src_stride, const int64_t* __restrict__ src_rows, int32_t V,
                       Rows rows, Commit commit, typename Dt<T>::Bits fill, int32_t chunk,
                       int32_t chunks_per_row, StepScratch ws,
                       const int32_t* __restrict__ nrows) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ unsigned long long warp_q[kWarps];
  __shared__ uint32_t warps_done;
  // rows at or past a device-held row count are not part of this call
  if (nrows != nullptr && static_cast<int32_t>(blockIdx.x / chunks_per_row) >= *nrows) return;
  if (threadIdx.x == 0) warps_done = 0u;
  if constexpr (kVec) fill_init<T>(smem, fill);
  __syncthreads();
  const int32_t row = blockIdx.x / chunks_per_row;
  const int32_t c0 = (blockIdx.x - row * chunks_per_row) * chunk;
  const WarpShare sh = warp_share<T, kVec>(c0, min(V, c0 + chunk));
  const RowInfo info = rows(row);
  ArgState st;
  bool issued = false;
  T* rowp = logits != nullptr ? logits + row * row_stride : nullptr;
  const S* srow;
  if constexpr (kInPlace) {
    srow = rowp;
  } else {
    srow = src + (src_rows != nullptr ? src_rows[row] : static_cast<int64_t>(row)) * src_stride;
  }
  constexpr bool kStaged = staged_path<kVec, kInPlace, Rows>();
  static_assert(!kStaged || Commit::kSmemBytes <= kStageWarpBytes,
                "a commit fits one warp's stage slice");
  if constexpr (kStaged) {
    uint4* stage = reinterpret_cast<uint4*>(smem + kFillBytes +
                                            (threadIdx.x >> 5) * kStageWarpBytes);
    warp_span_staged<T, true>(rowp, sh.e0, sh.nt, sh.s0, sh.s1, info.brow, fill,
                              reinterpret_cast<const uint4*>(smem), stage, st, issued);
  } else {
    warp_span<T, S, kInPlace, kVec, true, Rows::kSoft>(rowp, srow, sh.e0, sh.nt, sh.s0,
                                                       sh.s1, info.brow, fill,
                                                       reinterpret_cast<const uint4*>(smem),
                                                       info.lrow, rows_alpha(rows), st, issued);
  }
  // Two-level last-arriver merge, no barrier: the CTA's last warp (a shared
  // memory count) merges the CTA's 8 partials and takes part in the row's
  // count in global memory; the row's last CTA commits.
  const unsigned long long q = warp_max_u64(pack_arg(st.key, st.idx));
  const int32_t lane = threadIdx.x & 31;
  int32_t tok = -1;
  if (lane == 0) {
    warp_q[threadIdx.x >> 5] = q;
    __threadfence_block();
    if (atomicAdd(&warps_done, 1u) == kWarps - 1) {
      __threadfence_block();
      unsigned long long m = 0;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) {
        const unsigned long long x = *static_cast<volatile unsigned long long*>(&warp_q[i]);
        m = x > m ? x : m;
      }
      if (chunks_per_row == 1) {
        tok = unpack_idx(m);
      } else {
        atomicMax(ws.best + row, m);
        // acquire-release count: this CTA's maximum is visible before the
        // count moves on, and the last CTA sees every other CTA's maximum
        uint32_t arrived;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(arrived)
                     : "l"(ws.done + row)
                     : "memory");
        if (arrived == static_cast<uint32_t>(chunks_per_row - 1)) {
          const unsigned long long b = atomicExch(ws.best + row, 0ull);
          ws.done[row] = 0u;
          tok = unpack_idx(b);
        }
      }
    }
    if (issued) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
  }
  tok = __shfl_sync(kAll, tok, 0);
  // the commit's shared memory: after the fill buffer, or -- staged -- this
  // warp's own stage slice, whose loads were all consumed by its span
  uint8_t* csmem = kStaged ? smem + kFillBytes + (threadIdx.x >> 5) * kStageWarpBytes
                           : smem + kFillBytes;
  if (tok >= 0) commit(row, info, tok, csmem);
}

// Lets `kernel` use `bytes` of dynamic shared memory on the current device
// (needed above 48 KB); done once per kernel and device.
template <auto kernel>
bpd_status allow_smem(size_t bytes, const char* what) {
  if (bytes <= 48 * 1024) return BPD_OK;
  constexpr int kMaxDev = 64;
  static int done[kMaxDev] = {};  // 1 + the size set, per device
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev)
    return fail(BPD_ERR_CUDA, "%s: cannot query the current device", what);
  if (done[dev] == static_cast<int>(bytes) + 1) return BPD_OK;
  const cudaError_t e = cudaFuncSetAttribute(
      kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess)
    return fail(BPD_ERR_CUDA, "%s: shared memory size %zu: %s", what, bytes,
                cudaGetErrorString(e));
  done[dev] = static_cast<int>(bytes) + 1;
  return BPD_OK;
}

// ---------------------------------------------------------------------------
// Persistent fused step: a grid of resident CTAs whose WARPS take work items
// -- (row, segment of seg_tiles warp tiles) -- from an atomic queue. The CTA
// fills its shared fill buffer once for the whole launch; each warp fetches
// its next item index one item ahead and issues the loads of that item's
// row (Rows::pre) before it streams the current one, so the dependent chain
// of a row (slot -> state -> allow row) overlaps the streaming instead of
// preceding it. A row's pieces meet as in stream_step_kernel: one 64-bit
// atomicMax per piece and an acquire-release count; the warp that completes
// the row commits it. Nothing waits on another warp or CTA; the last warp to
// finish resets the queue (release fence before each warp's exit count).
//
// The last segment of a row also takes its ragged end (V mod TILE elements,
// one per lane). Segments past the row's tiles (chunks_per_row larger than
// the tile count) are empty pieces that still count.
#ifndef BPD_PERSIST
#define BPD_PERSIST 1
#endif
#ifndef BPD_PERSIST_BLOCKS
#define BPD_PERSIST_BLOCKS 5
#endif
#ifndef BPD_SEG_TILES
#define BPD_SEG_TILES 8
#endif

template <typename T, typename S, bool kInPlace, class Rows, class Commit>
__global__ void __launch_bounds__(kThreads, BPD_PERSIST_BLOCKS)
    persist_step_kernel(T* __restrict__ logits, int64_t row_stride, const S* __restrict__ src,
                        int64_t src_stride, const int64_t* __restrict__ src_rows, int32_t V,
                        Rows rows, Commit commit, typename Dt<T>::Bits fill, int32_t seg_tiles,
                        int32_t segs_per_row, int32_t items, StepScratch ws,
                        const int32_t* __restrict__ nrows) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int32_t TILE = tile_elems<T>();
  fill_init<T>(smem, fill);
  __syncthreads();
  const uint4* sfill = reinterpret_cast<const uint4*>(smem);
  const int32_t lane = threadIdx.x & 31;
  uint8_t* csmem = smem + kFillBytes + (threadIdx.x >> 5) * Commit::kSmemBytes;
  const int32_t ntr = V / TILE;  // full warp tiles of a row
  uint32_t item = 0, nxt = 0;
  if (lane == 0) {
    item = atomicAdd(ws.queue, 1u);
    nxt = atomicAdd(ws.queue, 1u);
  }
  item = __shfl_sync(kAll, item, 0);
  nxt = __shfl_sync(kAll, nxt, 0);
  // with a device-held row count, only the items of rows below it
  const uint32_t nitems =
      nrows == nullptr
          ? static_cast<uint32_t>(items)
          : static_cast<uint32_t>(min(items, max(0, min(*nrows, items / segs_per_row)) *
                                                 segs_per_row));
  typename Rows::Pre pre{};
  if (item < nitems) pre = rows.pre(static_cast<int32_t>(item) / segs_per_row);
  bool any_issued = false;
  while (item < nitems) {
    const int32_t row = static_cast<int32_t>(item) / segs_per_row;
    const int32_t seg = static_cast<int32_t>(item) - row * segs_per_row;
    // the next item's row loads and the index after it: in flight while
    // this item streams
    typename Rows::Pre npre{};
    if (nxt < nitems) npre = rows.pre(static_cast<int32_t>(nxt) / segs_per_row);
    uint32_t after = 0;
    if (lane == 0 && nxt < nitems) after = atomicAdd(ws.queue, 1u);
    const RowInfo info = rows.info(row, pre);
    const int32_t t0 = seg * seg_tiles;
    const int32_t nt = max(0, min(seg_tiles, ntr - t0));
    const bool last = seg == segs_per_row - 1;
    const int32_t e0 = min(t0, ntr) * TILE;
    const int32_t s0 = ntr * TILE;
    const int32_t s1 = last ? V : s0;
    T* rowp = logits != nullptr ? logits + row * row_stride : nullptr;
    const S* srow;
    if constexpr (kInPlace) {
      srow = rowp;
    } else {
      srow = src + (src_rows != nullptr ? src_rows[row] : static_cast<int64_t>(row)) * src_stride;
    }
    ArgState st;
    bool issued = false;
    warp_span<T, S, kInPlace, true, true, Rows::kSoft>(rowp, srow, e0, nt, s0, s1, info.brow,
                                                        fill, sfill, info.lrow, rows_alpha(rows),
                                                        st, issued);
    any_issued = any_issued || issued;
    const unsigned long long q = warp_max_u64(pack_arg(st.key, st.idx));
    int32_t tok = -1;
    if (lane == 0) {
      if (segs_per_row == 1) {
        tok = unpack_idx(q);
      } else {
        atomicMax(ws.best + row, q);
        uint32_t arrived;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                     : "=r"(arrived)
                     : "l"(ws.done + row)
                     : "memory");
        if (arrived == static_cast<uint32_t>(segs_per_row - 1)) {
          const unsigned long long b = atomicExch(ws.best + row, 0ull);
          ws.done[row] = 0u;
          tok = unpack_idx(b);
        }
      }
      // bound the bulk stores this thread has in flight (their source is the
      // read-only fill buffer, so only the count matters)
      if (any_issued) asm volatile("cp.async.bulk.wait_group.read 8;" ::: "memory");
    }
    tok = __shfl_sync(kAll, tok, 0);
    if (tok >= 0) commit(row, info, tok, csmem);
    item = nxt;
    nxt = __shfl_sync(kAll, after, 0);
    pre = npre;
  }
  if (lane == 0) {
    if (any_issued) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    // every queue fetch of this warp is ordered before its exit count; the
    // last warp out sees all of them and clears the queue for the next launch
    __threadfence();
    uint32_t out;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(out)
                 : "l"(ws.queue + 1)
                 : "memory");
    if (out == gridDim.x * static_cast<uint32_t>(kWarps) - 1u) {
      ws.queue[0] = 0u;
      ws.queue[1] = 0u;
    }
  }
}

// Work layout of the persistent step: warp tiles per segment and segments
// per row. chunks_per_row > 0 sets the segment count; 0 picks BPD_SEG_TILES
// tiles per segment, halved for small batches until there are about 4 items
// per SM.
struct PersistLayout {
  int32_t seg_tiles, segs, items, grid;
};

template <typename T>
inline PersistLayout persist_layout(int32_t V, int32_t batch, int32_t chunks_per_row) {
  constexpr int32_t TILE = tile_elems<T>();
  const int32_t ntr = V / TILE;
  const int64_t sms = sm_count();
  PersistLayout L;
  if (chunks_per_row > 0) {
    L.segs = chunks_per_row;
    L.seg_tiles = max(1, (ntr + L.segs - 1) / L.segs);
  } else {
    L.seg_tiles = BPD_SEG_TILES;
    while (L.seg_tiles > 1 &&
           static_cast<int64_t>(batch) * ((ntr + L.seg_tiles - 1) / L.seg_tiles) < sms * 4)
      L.seg_tiles /= 2;
    L.segs = max(1, (ntr + L.seg_tiles - 1) / L.seg_tiles);
  }
  const int64_t items = static_cast<int64_t>(batch) * L.segs;
  L.items = items < 0x7FFFFFFF ? static_cast<int32_t>(items) : -1;
  L.grid = static_cast<int32_t>(std::min<int64_t>(sms * BPD_PERSIST_BLOCKS, std::max<int64_t>(items, 1)));
  return L;
}

template <typename T, typename S, bool kInPlace, class Rows, class Commit>
bpd_status launch_persist_step(T* out, int64_t out_stride, const S* src, int64_t src_stride,
                               const int64_t* src_rows, int32_t batch, int32_t V,
                               const Rows& rows, const Commit& commit,
                               typename Dt<T>::Bits fill, int32_t chunks_per_row,
                               const StepScratch& ws, cudaStream_t st, const char* what,
                               const int32_t* nrows = nullptr) {
  const PersistLayout L = persist_layout<T>(V, batch, chunks_per_row);
  if (L.items < 0) return fail(BPD_ERR_INVALID, "%s: batch too large", what);
  const size_t smem = static_cast<size_t>(kFillBytes) +
                      static_cast<size_t>(kWarps) * static_cast<size_t>(Commit::kSmemBytes);
  const bpd_status rc =
      allow_smem<persist_step_kernel<T, S, kInPlace, Rows, Commit>>(smem, what);
  if (rc) return rc;
  persist_step_kernel<T, S, kInPlace, Rows, Commit>
      <<<static_cast<unsigned>(L.grid), kThreads, smem, st>>>(
          out, out_stride, src, src_stride, src_rows, V, rows, commit, fill, L.seg_tiles, L.segs,
          L.items, ws, nrows);
  return check_launch(what);
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
  const int32_t chunk = stream_chunk<T>(V, 0, batch);
  const int32_t chunks = (V + chunk - 1) / chunk;
  const int64_t grid = static_cast<int64_t>(batch) * chunks;
  if (grid >= 0x7FFFFFFF) return fail(BPD_ERR_INVALID, "%s: batch too large", what);
  const auto fill = Dt<T>::from_float_host(neg_inf);
  T* lg = static_cast<T*>(logits);
  if (vec_ok<Rows>(logits, row_stride, sizeof(T), V)) {
    constexpr size_t smem = stream_smem_bytes<staged_path<true, true, Rows>()>(0);
    const bpd_status rc = allow_smem<stream_apply_kernel<T, true, Rows>>(smem, what);
    if (rc) return rc;
    stream_apply_kernel<T, true, Rows><<<static_cast<unsigned>(grid), kThreads, smem, st>>>(
        lg, row_stride, V, rows, fill, chunk, chunks);
  } else {
    stream_apply_kernel<T, false, Rows><<<static_cast<unsigned>(grid), kThreads, 0, st>>>(
        lg, row_stride, V, rows, fill, chunk, chunks);
  }
  return check_launch(what);
}

template <typename T, class Rows, class Commit>
bpd_status launch_stream_step(void* logits, int64_t row_stride, int32_t batch, int32_t V,
                              const Rows& rows, const Commit& commit, float neg_inf,
                              int32_t chunks_per_row, void* scratch, cudaStream_t st,
                              const char* what) {
  if (scratch == nullptr) return fail(BPD_ERR_INVALID, "%s: null step scratch", what);
  if (!aligned16(scratch))
    return fail(BPD_ERR_INVALID, "%s: step scratch not 16-byte aligned", what);
  const int32_t chunk = stream_chunk<T>(V, chunks_per_row, batch);
  const int32_t cpr = (V + chunk - 1) / chunk;
  const int64_t grid = static_cast<int64_t>(batch) * cpr;
  if (grid >= 0x7FFFFFFF) return fail(BPD_ERR_INVALID, "%s: batch too large", what);
  const auto fill = Dt<T>::from_float_host(neg_inf);
  const StepScratch ws = step_scratch_view(scratch, batch);
  T* lg = static_cast<T*>(logits);
  const size_t smem = kFillBytes + Commit::kSmemBytes;
  if (BPD_PERSIST && vec_ok<Rows>(logits, row_stride, sizeof(T), V)) {
    return launch_persist_step<T, T, true, Rows, Commit>(lg, row_stride, lg, row_stride, nullptr,
                                                         batch, V, rows, commit, fill,
                                                         chunks_per_row, ws, st, what);
  }
  if (vec_ok<Rows>(logits, row_stride, sizeof(T), V)) {
    constexpr size_t vsmem =
        stream_smem_bytes<staged_path<true, true, Rows>()>(Commit::kSmemBytes);
    const bpd_status rc =
        allow_smem<stream_step_kernel<T, T, true, true, Rows, Commit>>(vsmem, what);
    if (rc) return rc;
    stream_step_kernel<T, T, true, true, Rows, Commit>
        <<<static_cast<unsigned>(grid), kThreads, vsmem, st>>>(lg, row_stride, lg, row_stride,
                                                                nullptr, V, rows, commit, fill,
                                                                chunk, cpr, ws, nullptr);
  } else {
    stream_step_kernel<T, T, true, false, Rows, Commit>
        <<<static_cast<unsigned>(grid), kThreads, smem, st>>>(lg, row_stride, lg, row_stride,
                                                               nullptr, V, rows, commit, fill,
                                                               chunk, cpr, ws, nullptr);
  }
  return check_launch(what);
}

// The fused step on fp32 working values read from a source of type S
// (gathered through `src_rows`, may be nullptr), written to `out` (fp32,
// may be nullptr: tokens and commits only).
template <typename S, class Rows, class Commit>
bpd_status launch_stream_step_src(const void* src, int64_t src_stride, const int64_t* src_rows,
                                  float* out, int64_t out_stride, int32_t batch, int32_t V,
                                  const Rows& rows, const Commit& commit, float neg_inf,
                                  int32_t chunks_per_row, void* scratch, cudaStream_t st,
                                  const char* what, const int32_t* nrows = nullptr) {
  if (scratch == nullptr) return fail(BPD_ERR_INVALID, "%s: null step scratch", what);
  if (!aligned16(scratch))
    return fail(BPD_ERR_INVALID, "%s: step scratch not 16-byte aligned", what);
  const int32_t chunk = stream_chunk<float>(V, chunks_per_row, batch);
  const int32_t cpr = (V + chunk - 1) / chunk;
  const int64_t grid = static_cast<int64_t>(batch) * cpr;
  if (grid >= 0x7FFFFFFF) return fail(BPD_ERR_INVALID, "%s: batch too large", what);
  const auto fill = Dt<float>::from_float_host(neg_inf);
  const StepScratch ws = step_scratch_view(scratch, batch);
  const size_t smem = kFillBytes + Commit::kSmemBytes;
  const bool vec = rows_aligned(src, src_stride, sizeof(S)) &&
                   (out == nullptr || rows_aligned(out, out_stride, sizeof(float))) &&
                   (!Rows::kSoft || V % 4 == 0);
  const S* sp = static_cast<const S*>(src);
  if (BPD_PERSIST && vec) {
    return launch_persist_step<float, S, false, Rows, Commit>(out, out_stride, sp, src_stride,
                                                              src_rows, batch, V, rows, commit,
                                                              fill, chunks_per_row, ws, st, what,
                                                              nrows);
  }
  if (vec) {
    stream_step_kernel<float, S, false, true, Rows, Commit>
        <<<static_cast<unsigned>(grid), kThreads, smem, st>>>(out, out_stride, sp, src_stride,
                                                               src_rows, V, rows, commit, fill,
                                                               chunk, cpr, ws, nrows);
  } else {
    stream_step_kernel<float, S, false, false, Rows, Commit>
        <<<static_cast<unsigned>(grid), kThreads, smem, st>>>(out, out_stride, sp, src_stride,
                                                               src_rows, V, rows, commit, fill,
                                                               chunk, cpr, ws, nrows);
  }
  return check_launch(what);
}

}  // namespace bpd
