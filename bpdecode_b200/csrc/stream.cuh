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

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kVPT = 4;  // 16-byte vectors per lane per warp tile
constexpr unsigned kAll = 0xFFFFFFFFu;

template <typename T>
constexpr int tile_elems() {
  return 32 * kVPT * Dt<T>::kPerVec;
}

// Running first-maximal element of a thread's share of a masked row.
struct ArgState {
  uint32_t key = 0;      // order_key of the best value seen (0 = none yet)
  int32_t idx = INT_MAX; // its index (the first one with that key)
};

// Key of the largest element of a 16-byte vector (NaN is the largest).
template <typename T>
__device__ __forceinline__ uint32_t vec_max_key(const uint4& v) {
  if constexpr (sizeof(typename Dt<T>::Bits) == 4) {
    const uint32_t a = max(order_key(__uint_as_float(v.x)), order_key(__uint_as_float(v.y)));
    const uint32_t b = max(order_key(__uint_as_float(v.z)), order_key(__uint_as_float(v.w)));
    return max(a, b);
  } else if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
    const __nv_bfloat162 m = __hmax2_nan(__hmax2_nan(p[0], p[1]), __hmax2_nan(p[2], p[3]));
    return max(order_key(__low2float(m)), order_key(__high2float(m)));
  } else {
    const __half2* p = reinterpret_cast<const __half2*>(&v);
    const __half2 m = __hmax2_nan(__hmax2_nan(p[0], p[1]), __hmax2_nan(p[2], p[3]));
    return max(order_key(__low2float(m)), order_key(__high2float(m)));
  }
}

// Fold the vector starting at element e0 into the running best: only a vector
// whose maximum beats the best so far is searched for its first maximal lane.
template <typename T>
__device__ __forceinline__ void arg_vec(ArgState& st, const uint4& v, int32_t e0) {
  const uint32_t k = vec_max_key<T>(v);
  if (k > st.key) {
    int32_t first = 0;
#pragma unroll
    for (int i = Dt<T>::kPerVec - 1; i >= 0; --i)
      if (order_key(Dt<T>::to_float(vec_get<T>(v, i))) == k) first = i;
    st.key = k;
    st.idx = e0 + first;
  }
}

__device__ __forceinline__ void arg_one(ArgState& st, uint32_t k, int32_t idx) {
  if (k > st.key) {
    st.key = k;
    st.idx = idx;
  }
}

// Masks [c0, c1) of `row` (c0 a multiple of the warp tile, so allow words line
// up) against allow row `brow` (nullptr = reject everything). With kArgmax the
// thread also tracks the first maximal element of the masked row (rejected
// elements count with the fill value, exactly as torch.argmax sees the row).
// Elements are visited in increasing order per thread, so a strict `>` keeps
// the first occurrence.
template <typename T, bool kVec, bool kArgmax>
__device__ __forceinline__ void mask_range(T* __restrict__ row, int32_t c0, int32_t c1,
                                           const uint32_t* __restrict__ brow,
                                           typename Dt<T>::Bits fill, ArgState& st) {
  using Bits = typename Dt<T>::Bits;
  constexpr int EPV = Dt<T>::kPerVec;
  constexpr int TILE = tile_elems<T>();
  constexpr int WPT = TILE / 32;  // allow words per warp tile
  constexpr uint32_t FULL = (1u << EPV) - 1u;
  const int32_t lane = threadIdx.x & 31;
  const int32_t warp = threadIdx.x >> 5;
  const uint32_t fill_key = kArgmax ? order_key(Dt<T>::to_float(fill)) : 0u;
  int32_t vend = c0;
  if constexpr (kVec) {
    const int32_t ntiles = c1 > c0 ? (c1 - c0) / TILE : 0;
    vend = c0 + ntiles * TILE;
    // the allow word of the next tile is loaded while this tile streams
    uint32_t w_next = 0;
    if (brow != nullptr && lane < WPT && warp < ntiles) w_next = __ldg(brow + ((c0 + warp * TILE) >> 5) + lane);
    for (int32_t ti = warp; ti < ntiles; ti += kWarps) {
      const int32_t tb = c0 + ti * TILE;
      const uint32_t w = w_next;
      if (brow != nullptr && lane < WPT && ti + kWarps < ntiles)
        w_next = __ldg(brow + ((tb + kWarps * TILE) >> 5) + lane);
      uint32_t bits[kVPT];
#pragma unroll
      for (int j = 0; j < kVPT; ++j) {
        const int v = lane + 32 * j;
        const uint32_t word = __shfl_sync(kAll, w, (v * EPV) >> 5);
        bits[j] = (word >> ((v * EPV) & 31)) & FULL;
      }
      uint4* base = reinterpret_cast<uint4*>(row + tb);
      uint4 val[kVPT];
#pragma unroll
      for (int j = 0; j < kVPT; ++j) {
        const bool need = kArgmax ? (bits[j] != 0u) : (bits[j] != 0u && bits[j] != FULL);
        if (need) val[j] = __ldcs(base + lane + 32 * j);
      }
#pragma unroll
      for (int j = 0; j < kVPT; ++j) {
        const int32_t e0 = tb + (lane + 32 * j) * EPV;
        if (bits[j] == FULL) {
          if constexpr (kArgmax) arg_vec<T>(st, val[j], e0);
        } else if (bits[j] == 0u) {
          __stcs(base + lane + 32 * j, vec_splat<T>(fill));
          if constexpr (kArgmax) arg_one(st, fill_key, e0);
        } else {
          const uint4 out = vec_blend<T>(val[j], bits[j], fill);
          __stcs(base + lane + 32 * j, out);
          if constexpr (kArgmax) arg_vec<T>(st, out, e0);
        }
      }
    }
  }
  Bits* rb = reinterpret_cast<Bits*>(row);
  for (int32_t e = vend + static_cast<int32_t>(threadIdx.x); e < c1; e += kThreads) {
    const bool allowed = brow != nullptr && ((__ldg(brow + (e >> 5)) >> (e & 31)) & 1u);
    if (allowed) {
      if constexpr (kArgmax) arg_one(st, order_key(Dt<T>::to_float(rb[e])), e);
    } else {
      rb[e] = fill;
      if constexpr (kArgmax) arg_one(st, fill_key, e);
    }
  }
}

}  // namespace bpd
