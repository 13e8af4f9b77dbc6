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

// Warp tiles whose allow words a warp loads at once (8, with the L2 warm-up,
// spilled registers: config-2 step 97-99 against 82-84 us).
#ifndef BPD_GROUP_TILES
#define BPD_GROUP_TILES 4
#endif
constexpr int kGroupTiles = BPD_GROUP_TILES;

// Cache policy of the logits stream: 0 = streaming (evict-first) loads and
// stores, 1 = loads and stores cached at L2 only (.cg). .cg measured 2 %
// faster on the config-2 step (86.7 against 88.4 µs per step over the first
// 20 steps of a generation, 65.1 against 66.3 over 128; same-box A/B).
#ifndef BPD_STREAM_CG
#define BPD_STREAM_CG 1
#endif

template <typename V>
__device__ __forceinline__ V ld_stream(const V* p) {
  if constexpr (BPD_STREAM_CG) {
    return __ldcg(p);
  } else {
    return __ldcs(p);
  }
}

__device__ __forceinline__ void st_stream(uint4* p, const uint4& v) {
  if constexpr (BPD_STREAM_CG) {
    __stcg(p, v);
  } else {
    __stcs(p, v);
  }
}

// The 16-byte vector of working type T at element e0 of a source row of type
// S: the same bits when S == T, else (T = float) EPV elements of S widened.
template <typename T, typename S>
__device__ __forceinline__ uint4 load_src(const S* __restrict__ srow, int32_t e0) {
  if constexpr (std::is_same_v<S, T>) {
    return ld_stream(reinterpret_cast<const uint4*>(srow + e0));
  } else {
    static_assert(std::is_same_v<T, float> && sizeof(S) == 2, "fp32 from 16-bit sources");
    const uint2 h = ld_stream(reinterpret_cast<const uint2*>(srow + e0));
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

// L2 warm-up of a group's later live tiles, issued as soon as the group's
// allow words are known, so their DRAM reads overlap the first live tile
// instead of starting one tile after another: 0 = off, 1 = per lane, the
// vectors the tile loop will load (prefetch.global.L2), 2 = the whole tile in
// one bulk prefetch by one lane (cp.async.bulk.prefetch.L2), 3 = mode 1 for
// in-place spans and mode 2 for spans that read another buffer. Same-box A/B
// against 0: mode 3 takes the config-2 fused step from 87.9 to 82.8 us over
// the first 20 steps of a generation (62.4 -> 61.4 over 128), the tokens-only
// step from 63.0 to 58.9 us, the config-3 fp32 step from 74.3 to 71.0 us; the
// PDA config-4 step, the soft step and config 5 are unchanged. Mode 1 alone
// made the tokens-only step 2 % slower, mode 2 alone the fused step 1 %
// slower than mode 3 (bulk prefetches also fetch the rejected vectors that
// the in-place step writes without reading).
#ifndef BPD_L2_PREFETCH
#define BPD_L2_PREFETCH 3
#endif

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// The same with evict-last priority (the soft step's lookahead rows, which
// rows in the same state share).
__device__ __forceinline__ void prefetch_l2_keep(const void* p) {
  asm volatile("prefetch.global.L2::evict_last [%0];" ::"l"(p));
}

// Soft spans: 0 = no L2 warm-up, 1 = per lane (logits and biases of every
// vector with an allowed token), 2 = whole tiles by one lane per tile, 3 =
// mode 1 for in-place spans, none for spans that read another buffer.
// Same-box A/B against 0: mode 1 takes the in-place fp32 soft step (1024
// rows) from 122.2 to 118.6 us but the config-5 loop, whose soft step reads
// bf16 model logits into an fp32 result, from 127.4 to 137.3 us; mode 2 is
// slower on both (124.3, 129.2).
#ifndef BPD_SOFT_PREFETCH
#define BPD_SOFT_PREFETCH 3
#endif

// p 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
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
  constexpr int WPT = TILE / 32;  // allow words per warp tile
  constexpr uint32_t FULL = (1u << EPV) - 1u;
  const int32_t lane = threadIdx.x & 31;
  // L2 warm-up mode of this span (BPD_L2_PREFETCH 3: per lane in place,
  // whole tiles when the values come from another buffer)
  constexpr int kPrefetch =
      BPD_L2_PREFETCH == 3 ? (kInPlace ? 1 : 2) : BPD_L2_PREFETCH;
  int32_t fill_first = INT_MAX;  // lowest index this lane wrote `fill` to
  VecArg va;
  if constexpr (kVec) {
    const int32_t ntiles = nt;
    for (int32_t g0 = 0; g0 < ntiles; g0 += kGroupTiles) {
      uint32_t w[kGroupTiles];
#pragma unroll
      for (int t = 0; t < kGroupTiles; ++t) {
        w[t] = 0u;
        if (brow != nullptr && g0 + t < ntiles && lane < WPT)
          w[t] = __ldg(brow + ((e0 + (g0 + t) * TILE) >> 5) + lane);
      }
      uint32_t live = 0u;
#pragma unroll
      for (int t = 0; t < kGroupTiles; ++t)
        live |= (__any_sync(kAll, w[t] != 0u) ? 1u : 0u) << t;
      constexpr int kSoftPrefetch =
          BPD_SOFT_PREFETCH == 3 ? (kInPlace ? 1 : 0) : BPD_SOFT_PREFETCH;
      if constexpr (kSoft && kSoftPrefetch != 0) {
        // soft spans load a tile's vectors a group at a time, so every live
        // tile is warmed, logits and lookahead biases alike
        if constexpr (kSoftPrefetch == 1) {
#pragma unroll
          for (int t = 0; t < kGroupTiles; ++t) {
            if (((live >> t) & 1u) == 0u) continue;
            const int32_t tb = e0 + (g0 + t) * TILE;
#pragma unroll
            for (int j = 0; j < kVPT; ++j) {
              if (tile_bits<T>(w[t], lane, j) == 0u) continue;
              const int32_t e = tb + (lane + 32 * j) * EPV;
              prefetch_l2(srow + e);
              prefetch_l2_keep(lrow + e);
            }
          }
        } else {
          if (lane < kGroupTiles && ((live >> lane) & 1u) != 0u) {
            const int32_t tb = e0 + (g0 + lane) * TILE;
            bulk_prefetch_l2(srow + tb,
                             static_cast<uint32_t>(TILE * static_cast<int32_t>(sizeof(S))));
            bulk_prefetch_l2(lrow + tb, static_cast<uint32_t>(TILE * 4));
          }
        }
      }
      if constexpr (!kSoft && BPD_PIPELINE && kPrefetch != 0) {
        // every live tile after the first: the first is loaded right away
        const uint32_t later = live & (live - 1u);
        if constexpr (kPrefetch == 1) {
#pragma unroll
          for (int t = 1; t < kGroupTiles; ++t) {
            if (((later >> t) & 1u) == 0u) continue;
            const int32_t tb = e0 + (g0 + t) * TILE;
#pragma unroll
            for (int j = 0; j < kVPT; ++j) {
              const uint32_t b = tile_bits<T>(w[t], lane, j);
              const bool need = (kArgmax || !kInPlace) ? (b != 0u) : (b != 0u && b != FULL);
              if (need) prefetch_l2(srow + tb + (lane + 32 * j) * EPV);
            }
          }
        } else {
          if (lane < kGroupTiles && ((later >> lane) & 1u) != 0u)
            bulk_prefetch_l2(srow + e0 + (g0 + lane) * TILE,
                             static_cast<uint32_t>(TILE * static_cast<int32_t>(sizeof(S))));
        }
      }
      const int32_t ng = min(kGroupTiles, ntiles - g0);
      uint32_t dead = ((1u << ng) - 1u) & ~live;
      if constexpr (sizeof(Bits) == 4) {
        // fp32: only a whole dead group goes out as one bulk store; dead
        // tiles among live ones take plain stores with them (-4 % on the
        // PDA step, neutral on the soft step; 16-bit rows keep every dead
        // tile on the bulk engine, which is faster there)
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
            if (row != nullptr && (!kInPlace || b != FULL)) st_stream(base + lane + 32 * j, out);
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
              st_stream(base + lane + 32 * j, out);
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

// Warp tiles each warp streams per CTA when the caller leaves the chunk to
// stream_chunk (a Rows type may ask for another count).
#ifndef BPD_TILES_PER_WARP
#define BPD_TILES_PER_WARP 4
#endif

struct DenseRows {
  static constexpr bool kSoft = false;
  static constexpr int kTilesPerWarp = BPD_TILES_PER_WARP;
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
// The in-place fused (non-soft) step then went to 64 registers (4 CTAs per
// SM): -1 % on the config-2 step with the .cg stream (85.8 against 86.8 µs
// over the first 20 steps of a generation; 6 CTAs per SM +8 %); the step on
// values read from another buffer (the *_from entry points) stays at 5 CTAs
// per SM, where 4 cost it 13 % (74.5 against 66.0 µs, tokens-only config 2).
#ifndef BPD_APPLY_MIN_BLOCKS
#define BPD_APPLY_MIN_BLOCKS 5
#endif
#ifndef BPD_STEP_MIN_BLOCKS
#define BPD_STEP_MIN_BLOCKS 4
#endif
#ifndef BPD_STEP_FROM_MIN_BLOCKS
#define BPD_STEP_FROM_MIN_BLOCKS 5
#endif
#ifndef BPD_SOFT_STEP_MIN_BLOCKS
#define BPD_SOFT_STEP_MIN_BLOCKS 5
#endif

// Chunk of one CTA: `chunks_per_row` CTAs per row when the caller asks for
// it, else `tiles_per_warp` warp tiles per warp (the Rows type's count).
// Always a multiple of kWarps warp tiles, so every warp span starts on a tile.
//
// With `batch` given, small batches are cut finer (down to one warp tile per
// warp) until the grid has about one CTA per SM, so a step over a handful of
// rows is not a few CTAs working through their tiles one after another
// (B = 1, V = 128,256: 13.9 -> 11.9 us per step replayed from a graph).
template <typename T>
inline int32_t stream_chunk(int32_t V, int32_t chunks_per_row, int32_t batch = 0,
                            int32_t tiles_per_warp = BPD_TILES_PER_WARP) {
  constexpr int32_t UNIT = tile_elems<T>() * kWarps;
  if (chunks_per_row <= 0) {
    int32_t tpw = tiles_per_warp;
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
__global__ void __launch_bounds__(kThreads, BPD_APPLY_MIN_BLOCKS)
    stream_apply_kernel(T* __restrict__ logits, int64_t row_stride, int32_t V, Rows rows,
                        typename Dt<T>::Bits fill, int32_t chunk, int32_t chunks_per_row) {
  extern __shared__ __align__(16) uint8_t smem[];
  if constexpr (kVec) {
    fill_init<T>(smem, fill);
    __syncthreads();
  }
  pdl_trigger();
  pdl_wait();  // the rows' states / allow rows come from the kernels before
  const int32_t row = blockIdx.x / chunks_per_row;
  const int32_t c0 = (blockIdx.x - row * chunks_per_row) * chunk;
  const WarpShare ws = warp_share<T, kVec>(c0, min(V, c0 + chunk));
  const RowInfo info = rows(row);
  ArgState st;
  bool issued = false;
  T* rowp = logits + row * row_stride;
  warp_span<T, T, true, kVec, false, Rows::kSoft>(rowp, rowp, ws.e0, ws.nt, ws.s0,
                                                  ws.s1, info.brow, fill,
                                                  reinterpret_cast<const uint4*>(smem), info.lrow,
                                                  rows_alpha(rows), st, issued);
  if (issued) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Device scratch of the fused step: per row the best packed (key, ~index) so
// far and the number of warps done. It must be zero before a launch; every
// launch that runs to completion leaves it zero again (the row's last warp
// clears it).
struct StepScratch {
  unsigned long long* best;  // [batch]
  uint32_t* done;            // [batch]
};

constexpr size_t step_scratch_bytes(int32_t batch) {
  return align256(sizeof(unsigned long long) * static_cast<size_t>(batch)) +
         align256(sizeof(uint32_t) * static_cast<size_t>(batch));
}

inline StepScratch step_scratch_view(void* base, int32_t batch) {
  char* p = static_cast<char*>(base);
  StepScratch s;
  s.best = reinterpret_cast<unsigned long long*>(p);
  s.done = reinterpret_cast<uint32_t*>(
      p + align256(sizeof(unsigned long long) * static_cast<size_t>(batch)));
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
                                  : kInPlace  ? BPD_STEP_MIN_BLOCKS
                                              : BPD_STEP_FROM_MIN_BLOCKS)
    stream_step_kernel(T* __restrict__ logits, int64_t row_stride, const S* __restrict__ src,
                       int64_t src_stride, const int64_t* __restrict__ src_rows, int32_t V,
                       Rows rows, Commit commit, typename Dt<T>::Bits fill, int32_t chunk,
                       int32_t chunks_per_row, StepScratch ws,
                       const int32_t* __restrict__ nrows) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ unsigned long long warp_q[kWarps];
  __shared__ uint32_t warps_done;
  if (threadIdx.x == 0) warps_done = 0u;
  if constexpr (kVec) fill_init<T>(smem, fill);
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // states, allow rows and the row count come from the kernels before
  // rows at or past a device-held row count are not part of this call (the
  // *_from_n entry points; the in-place steps never take one); the whole CTA
  // leaves together, and no barrier follows
  if constexpr (!kInPlace) {
    if (nrows != nullptr && static_cast<int32_t>(blockIdx.x / chunks_per_row) >= *nrows) return;
  }
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
  warp_span<T, S, kInPlace, kVec, true, Rows::kSoft>(rowp, srow, sh.e0, sh.nt, sh.s0,
                                                     sh.s1, info.brow, fill,
                                                     reinterpret_cast<const uint4*>(smem),
                                                     info.lrow, rows_alpha(rows), st, issued);
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
  if (tok >= 0) commit(row, info, tok, smem + kFillBytes);
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
  const int32_t chunk = stream_chunk<T>(V, 0, batch, Rows::kTilesPerWarp);
  const int32_t chunks = (V + chunk - 1) / chunk;
  const int64_t grid = static_cast<int64_t>(batch) * chunks;
  if (grid >= 0x7FFFFFFF) return fail(BPD_ERR_INVALID, "%s: batch too large", what);
  const auto fill = Dt<T>::from_float_host(neg_inf);
  T* lg = static_cast<T*>(logits);
  if (vec_ok<Rows>(logits, row_stride, sizeof(T), V)) {
    const cudaError_t e = launch_pdl(stream_apply_kernel<T, true, Rows>,
                                     dim3(static_cast<unsigned>(grid)), dim3(kThreads), kFillBytes,
                                     st, lg, row_stride, V, rows, fill, chunk, chunks);
    if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  } else {
    const cudaError_t e = launch_pdl(stream_apply_kernel<T, false, Rows>,
                                     dim3(static_cast<unsigned>(grid)), dim3(kThreads), 0, st, lg,
                                     row_stride, V, rows, fill, chunk, chunks);
    if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
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
  const int32_t chunk = stream_chunk<T>(V, chunks_per_row, batch, Rows::kTilesPerWarp);
  const int32_t cpr = (V + chunk - 1) / chunk;
  const int64_t grid = static_cast<int64_t>(batch) * cpr;
  if (grid >= 0x7FFFFFFF) return fail(BPD_ERR_INVALID, "%s: batch too large", what);
  const auto fill = Dt<T>::from_float_host(neg_inf);
  const StepScratch ws = step_scratch_view(scratch, batch);
  T* lg = static_cast<T*>(logits);
  const size_t smem = kFillBytes + Commit::kSmemBytes;
  const int64_t* no_rows = nullptr;
  const int32_t* no_count = nullptr;
  cudaError_t e;
  if (vec_ok<Rows>(logits, row_stride, sizeof(T), V)) {
    e = launch_pdl(stream_step_kernel<T, T, true, true, Rows, Commit>,
                   dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem, st, lg, row_stride,
                   static_cast<const T*>(lg), row_stride, no_rows, V, rows, commit, fill, chunk,
                   cpr, ws, no_count);
  } else {
    e = launch_pdl(stream_step_kernel<T, T, true, false, Rows, Commit>,
                   dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem, st, lg, row_stride,
                   static_cast<const T*>(lg), row_stride, no_rows, V, rows, commit, fill, chunk,
                   cpr, ws, no_count);
  }
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
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
  const int32_t chunk = stream_chunk<float>(V, chunks_per_row, batch, Rows::kTilesPerWarp);
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
  cudaError_t e;
  if (vec) {
    e = launch_pdl(stream_step_kernel<float, S, false, true, Rows, Commit>,
                   dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem, st, out, out_stride,
                   sp, src_stride, src_rows, V, rows, commit, fill, chunk, cpr, ws, nrows);
  } else {
    e = launch_pdl(stream_step_kernel<float, S, false, false, Rows, Commit>,
                   dim3(static_cast<unsigned>(grid)), dim3(kThreads), smem, st, out, out_stride,
                   sp, src_stride, src_rows, V, rows, commit, fill, chunk, cpr, ws, nrows);
  }
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

}  // namespace bpd
