// Shared helpers of the sm_100a kernels: error reporting for the C ABI,
// 16-byte vector access, logits dtype traits and the argmax ordering key.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "bpdecode_b200.h"

namespace bpd {

// Records a message for bpd_last_error() on this host thread and returns code.
bpd_status fail(bpd_status code, const char* fmt, ...);

// Checks the launch that was just enqueued.
bpd_status check_launch(const char* what);

// Multiprocessor count of the current device (cached per device).
int32_t sm_count();

inline cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

#define BPD_REQUIRE(cond, ...)                                   \
  do {                                                           \
    if (!(cond)) return ::bpd::fail(BPD_ERR_INVALID, __VA_ARGS__); \
  } while (0)

// ---------------------------------------------------------------------------
// logits dtype traits: 16-byte vectors hold kPerVec elements; `Bits` is the
// raw storage word of one element.
template <typename T>
struct Dt;

template <>
struct Dt<float> {
  using Bits = uint32_t;
  static constexpr int kPerVec = 4;
  __host__ __device__ static float to_float(Bits b) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(b);
#else
    float f;
    __builtin_memcpy(&f, &b, 4);
    return f;
#endif
  }
  static Bits from_float_host(float f) {
    Bits b;
    __builtin_memcpy(&b, &f, 4);
    return b;
  }
  __device__ static Bits from_float_dev(float f) { return __float_as_uint(f); }
};

template <>
struct Dt<__nv_bfloat16> {
  using Bits = uint16_t;
  static constexpr int kPerVec = 8;
  __device__ static float to_float(Bits b) { return __uint_as_float(uint32_t(b) << 16); }
  static Bits from_float_host(float f) {
    __nv_bfloat16 h = __float2bfloat16_rn(f);
    Bits b;
    __builtin_memcpy(&b, &h, 2);
    return b;
  }
  __device__ static Bits from_float_dev(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
};

template <>
struct Dt<__half> {
  using Bits = uint16_t;
  static constexpr int kPerVec = 8;
  __device__ static float to_float(Bits b) { return __half2float(__ushort_as_half(b)); }
  static Bits from_float_host(float f) {
    __half h = __float2half_rn(f);
    Bits b;
    __builtin_memcpy(&b, &h, 2);
    return b;
  }
  __device__ static Bits from_float_dev(float f) { return __half_as_ushort(__float2half_rn(f)); }
};

// Calls f(T{}) with T the logits element type of `dtype` (BPD_F32 / BPD_BF16 /
// BPD_F16), or fails with "<what>: unsupported <kind> dtype".
template <class F>
bpd_status with_dtype(int32_t dtype, const char* what, F&& f, const char* kind = "logits") {
  switch (dtype) {
    case BPD_F32:
      return f(float{});
    case BPD_BF16:
      return f(__nv_bfloat16{});
    case BPD_F16:
      return f(__half{});
    default:
      return fail(BPD_ERR_INVALID, "%s: unsupported %s dtype %d", what, kind, dtype);
  }
}

constexpr size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Programmatic dependent launch: the per-step kernels are launched with the
// programmatic-serialization attribute, start their grid's successor early
// (pdl_trigger) and wait for their predecessor to complete, with its memory
// visible, before their first global memory access (pdl_wait); only shared
// memory set-up comes before the wait. A dependent grid is scheduled only once
// every CTA of its predecessor has started, so CTAs blocked in the wait never
// keep a predecessor's CTAs off the SMs. Launched without the attribute (or
// after a kernel that never triggers) the wait returns at once.
#ifndef BPD_PDL
#define BPD_PDL 1
#endif

__device__ __forceinline__ void pdl_wait() {
  if constexpr (BPD_PDL) asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_trigger() {
  if constexpr (BPD_PDL) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... K, typename... A>
cudaError_t launch_pdl(void (*kernel)(K...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = BPD_PDL ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<A&&>(args)...);
  if (e != cudaSuccess) (void)cudaGetLastError();  // reported here, not by a later check
  return e;
}

__device__ __forceinline__ uint32_t vec_word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Element j (0 <= j < kPerVec) of a 16-byte vector (j is a compile-time
// constant after unrolling, so the selects fold away).
template <typename T>
__device__ __forceinline__ typename Dt<T>::Bits vec_get(const uint4& v, int j) {
  if constexpr (sizeof(typename Dt<T>::Bits) == 4) {
    return vec_word(v, j);
  } else {
    const uint32_t w = vec_word(v, j >> 1);
    return static_cast<uint16_t>((j & 1) ? (w >> 16) : (w & 0xFFFFu));
  }
}

// A vector with every element equal to `b`.
template <typename T>
__device__ __forceinline__ uint4 vec_splat(typename Dt<T>::Bits b) {
  uint32_t w;
  if constexpr (sizeof(typename Dt<T>::Bits) == 4) {
    w = b;
  } else {
    w = uint32_t(b) | (uint32_t(b) << 16);
  }
  return make_uint4(w, w, w, w);
}

// Blend: element j keeps `v` where bit j of `keep` is set, else `fill`.
template <typename T>
__device__ __forceinline__ uint4 vec_blend(const uint4& v, uint32_t keep, typename Dt<T>::Bits fill) {
  if constexpr (sizeof(typename Dt<T>::Bits) == 4) {
    return make_uint4((keep & 1) ? v.x : fill, (keep & 2) ? v.y : fill, (keep & 4) ? v.z : fill,
                      (keep & 8) ? v.w : fill);
  } else {
    // the two bits of word k move to bits 0 and 16 (t + (t << 15) cannot carry
    // for t < 256), and * 0xFFFF widens each to a 16-bit lane mask
    const uint32_t f2 = uint32_t(fill) | (uint32_t(fill) << 16);
    auto mix = [&](uint32_t w, uint32_t t) -> uint32_t {
      const uint32_t m = ((t * 0x8001u) & 0x10001u) * 0xFFFFu;
      return (w & m) | (f2 & ~m);
    };
    return make_uint4(mix(v.x, keep), mix(v.y, keep >> 2), mix(v.z, keep >> 4),
                      mix(v.w, keep >> 6));
  }
}

// Total order of float values for argmax: larger value -> larger key; NaN is
// the largest (torch.argmax treats NaN as maximal); -0.0 and +0.0 tie.
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0xFFFFFFFFu;
  if (f == 0.0f) f = 0.0f;
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// (key, index) packed so that the maximum prefers the larger key, then the
// smaller index -- the first maximal element, like torch.argmax.
__device__ __forceinline__ uint64_t pack_arg(uint32_t key, int32_t idx) {
  return (uint64_t(key) << 32) | uint64_t(~uint32_t(idx));
}
__device__ __forceinline__ int32_t unpack_idx(uint64_t p) { return int32_t(~uint32_t(p)); }

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

}  // namespace bpd
