// Pushdown-automaton (context-free grammar) kernels.
//
// Parity contract: the bounded config-set semantics of the reference's
// pda.hpp:95-258 -- push order, the 8-config / 32-frame caps, the `saturated`
// flag, the order-preserving dead-config prune and whole-struct copies -- so
// masks, ok flags and full 266-int config rows are identical.
//
// Design.
// * A config-set lives in shared memory and is worked on by ONE WARP: lane k
//   owns stack frame k (kPdaMaxDepth = 32 = warp width). Building a candidate
//   stack, comparing it against every existing config (one vote per config)
//   and pushing it are all single warp-wide steps instead of 32-iteration
//   loops over local memory.
// * Closure runs as a single in-order pass over the growing config list. The
//   reference runs rounds over [0, n) until no push succeeds; re-visiting an
//   already-processed config can neither push (its candidates are present, or
//   were dropped for a full set that never shrinks) nor change `saturated`
//   (already set), so one pass that keeps going until it reaches the end of
//   the list performs the same pushes in the same order.
// * Mask of a row = for every token, does its byte walk keep the set
//   non-empty. The walks go through a transition cache built on the device
//   (config-sets interned as nodes with 256 byte transitions, each computed
//   once by the bounded closure), so a token costs a few table reads once
//   its stretch of the grammar has been visited; without a memo, the first
//   bytes that keep each set alive are found first (256 warp walks) and only
//   longer tokens whose first byte survives are walked.
// * Mask memo in HBM, keyed by the config-set's live content (`saturated` and
//   words outside the live region do not affect the mask and are not part of
//   the key): an open-addressing table of {hash, canonical 266-int key, packed
//   allow row}. Rows of a step whose key is present reuse the stored row;
//   identical misses within one step are de-duplicated so each distinct
//   config-set is simulated once. The apply pass then streams logits exactly
//   like the dense path.
//
// Per mask call (all on the caller's stream, no host sync):
//   prologue_kernel (clears the call's workspace; the transition cache when
//   it filled up) -> lookup_kernel (memo probe, dedup, memo claim)
//   -> [first_byte_kernel, without a memo] -> compute_kernel (misses only; it
//   ends at once when every row hit) -> apply, or the fused step (apply +
//   argmax, and the warp that finishes a row advances its config-set by the
//   winning token).
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "stream.cuh"

namespace bpd {
namespace {

constexpr int MC = BPD_PDA_MAX_CONFIGS;
constexpr int MD = BPD_PDA_MAX_DEPTH;
constexpr int NCFG = BPD_PDA_CONFIG_INTS;
constexpr int kEps = 0, kByte = 1, kCall = 2;
constexpr int kProbe = 32;  // memo / dedup probe limit

static_assert(MD == 32, "one lane per stack frame");

__device__ __forceinline__ int32_t& n_of(int32_t* c) { return c[0]; }
__device__ __forceinline__ int32_t n_of(const int32_t* c) { return c[0]; }
__device__ __forceinline__ int32_t* st_of(int32_t* c, int i) { return c + 2 + MC + i * MD; }
__device__ __forceinline__ const int32_t* st_of(const int32_t* c, int i) {
  return c + 2 + MC + i * MD;
}

// Is a config equal to the candidate (depth cd >= 1; lane k holds frame k)
// in `c`? pda.hpp:102-108. Lane j < num_configs first checks config j's depth
// and top frame against the candidate's (one ballot); only the configs that
// pass are compared frame by frame.
__device__ __forceinline__ bool w_contains(const int32_t* c, int cd, int32_t v, int lane) {
  const int n = n_of(c);
  const int32_t top = __shfl_sync(kAll, v, cd - 1);
  const bool maybe = lane < n && c[2 + lane] == cd && st_of(c, lane)[cd - 1] == top;
  uint32_t cand = __ballot_sync(kAll, maybe);
  while (cand != 0u) {
    const int j = __ffs(cand) - 1;
    cand &= cand - 1u;
    const bool eq = lane >= cd || st_of(c, j)[lane] == v;
    if (__all_sync(kAll, eq)) return true;
  }
  return false;
}

// pda.hpp:111-121. Caller guarantees all lanes see the same `c` contents.
__device__ __forceinline__ bool w_push(int32_t* c, int cd, int32_t v, int lane) {
  const int n = n_of(c);
  if (n >= MC) {
    if (lane == 0) c[1] = 1;
    __syncwarp();
    return false;
  }
  if (lane < cd) st_of(c, n)[lane] = v;
  if (lane == 0) {
    c[2 + n] = cd;
    c[0] = n + 1;
  }
  __syncwarp();
  return true;
}

__device__ __forceinline__ void w_add(int32_t* c, int cd, int32_t v, int lane) {
  if (!w_contains(c, cd, v, lane)) w_push(c, cd, v, lane);
}

// pda.hpp:124-139 -- order-preserving compaction of configs whose top is live.
__device__ void w_prune(const bpd_pda_grammar& g, int32_t* c, int lane) {
  const int n = n_of(c);
  int out = 0;
  for (int i = 0; i < n; ++i) {
    const int d = c[2 + i];
    if (d <= 0) continue;
    if (!__ldg(g.live + st_of(c, i)[d - 1])) continue;
    if (out != i) {
      const int32_t v = lane < d ? st_of(c, i)[lane] : 0;
      if (lane < d) st_of(c, out)[lane] = v;
      if (lane == 0) c[2 + out] = d;
      __syncwarp();
    }
    ++out;
  }
  if (lane == 0) c[0] = out;
  __syncwarp();
}

// pda.hpp:150-198 as one in-order pass (see the file comment).
__device__ bool w_close(const bpd_pda_grammar& g, int32_t* c, int lane) {
  for (int i = 0; i < n_of(c); ++i) {
    const int d = c[2 + i];
    if (d <= 0) continue;
    const int32_t mine = lane < d ? st_of(c, i)[lane] : 0;
    const int32_t top = st_of(c, i)[d - 1];
    if (__ldg(g.accept + top) && d > 1) w_add(c, d - 1, mine, lane);  // pop
    const int eb = __ldg(g.edge_offsets + top);
    const int ee = __ldg(g.edge_offsets + top + 1);
    for (int e = eb; e < ee; ++e) {
      const int kind = __ldg(g.edge_kind + e);
      if (kind == kEps) {
        const int32_t v = lane == d - 1 ? __ldg(g.edge_dst + e) : mine;
        w_add(c, d, v, lane);
      } else if (kind == kCall) {
        if (d + 1 <= MD) {
          const int32_t v = lane == d - 1 ? __ldg(g.edge_dst + e)
                            : lane == d   ? __ldg(g.edge_callee + e)
                                          : mine;
          w_add(c, d + 1, v, lane);
        } else {
          if (lane == 0) c[1] = 1;
          __syncwarp();
        }
      }
    }
  }
  w_prune(g, c, lane);
  return n_of(c) > 0;
}

// pda.hpp:211-236: dst = close(byte-step of src). With kExact the whole 266
// words of dst are defined exactly as the reference's freshly zeroed `next`
// (needed when the row is written back); without it only the live region is
// meaningful, which is all a mask needs.
template <bool kExact>
__device__ bool w_advance_byte(const bpd_pda_grammar& g, const int32_t* src, int32_t* dst,
                               int byte, int lane) {
  if constexpr (kExact) {
    for (int k = lane; k < NCFG; k += 32) dst[k] = 0;
  } else {
    if (lane == 0) {
      dst[0] = 0;
      dst[1] = 0;
    }
  }
  __syncwarp();
  const int n = n_of(src);
  for (int i = 0; i < n; ++i) {
    const int d = src[2 + i];
    if (d <= 0) continue;
    const int32_t mine = lane < d ? st_of(src, i)[lane] : 0;
    const int32_t top = st_of(src, i)[d - 1];
    const int eb = __ldg(g.edge_offsets + top);
    const int ee = __ldg(g.edge_offsets + top + 1);
    for (int e = eb; e < ee; ++e) {
      if (__ldg(g.edge_kind + e) != kByte) continue;
      if (byte < __ldg(g.edge_lo + e) || byte > __ldg(g.edge_hi + e)) continue;
      const int32_t v = lane == d - 1 ? __ldg(g.edge_dst + e) : mine;
      w_add(dst, d, v, lane);
    }
  }
  if (lane == 0) dst[1] = (dst[1] || src[1]) ? 1 : 0;
  __syncwarp();
  return w_close(g, dst, lane);
}

// pda.hpp:238-244
__device__ __forceinline__ bool is_complete(const bpd_pda_grammar& g, const int32_t* c) {
  const int n = n_of(c);
  for (int i = 0; i < n; ++i)
    if (c[2 + i] == 1 && st_of(c, i)[0] == g.root_accept) return true;
  return false;
}

__device__ __forceinline__ void w_copy(int32_t* dst, const int32_t* src, int lane) {
  for (int k = lane; k < NCFG; k += 32) dst[k] = src[k];
  __syncwarp();
}

// ---------------------------------------------------------------------------
// Memo / workspace layout.

// Transition cache of the miss path: config-sets that token walks reach,
// interned as nodes (canonical content, as memo keys), each with its 256
// byte transitions filled in as walks need them. It turns the walks through
// regular stretches of a grammar (string bodies, numbers, keywords -- the
// regular sub-loops) into table walks, like a DFA's tok_next, while every
// transition is still the bounded closure of the reference on the node's
// exact content.
struct Nodes {
  unsigned long long* hash;  // [ncap] 0 = free, else (content hash | 1): slot claimed
  uint32_t* ready;           // [ncap] 1 once the slot's key is written
  int32_t* key;              // [ncap][NCFG] canonical config-sets
  int32_t* trans;            // [ncap][256] 0 unknown, 1 being computed, 2 the set dies,
                             //             3 + id: next node
  int32_t cap;               // power of two, 0 = none
  uint32_t* full;            // the memo header's "a node could not be interned" flag
};

struct Memo {
  uint32_t* epoch;  // header (256 B): [0] calls so far -- entries claimed by the
                    //     running call carry tag epoch + 1 and are skipped by its
                    //     own lookups; [1] set when a node could not be interned
                    //     (the table is full: the next call clears it);
                    //     [2] the call prologue's finished-CTA count
  uint32_t* tag;    // [cap] 0 = empty, else the claiming call's tag
  uint64_t* hash;   // [cap]
  int32_t* key;     // [cap][NCFG] canonical config-sets
  uint32_t* bits;   // [cap][ws] allow rows
  int32_t cap;      // power of two, 0 = no memo
  int32_t ws;       // words per allow row (multiple of 4)
  Nodes nodes;      // transition cache (kNodesPerEntry per memo entry)
};

// 16 nodes per memo entry: 64K nodes (~137 MB) at the default 4096 entries,
// room for a whole call of ~250 new config-sets with their walks' prefixes.
constexpr int32_t kNodesPerEntry = 16;
constexpr int kHdrNodesFull = 1, kHdrPrologueDone = 2;
#ifndef BPD_PDA_NODES
#define BPD_PDA_NODES 1  // 0: miss path without the transition cache (for comparisons)
#endif


constexpr int32_t words_stride(int32_t vocab) { return ((((vocab + 31) / 32) + 3) / 4) * 4; }

Memo memo_view(void* base, int32_t cap, int32_t vocab) {
  Memo m{};
  m.cap = base ? cap : 0;
  m.ws = words_stride(vocab);
  if (!base) return m;
  char* p = static_cast<char*>(base);
  m.epoch = reinterpret_cast<uint32_t*>(p);
  p += 256;
  m.tag = reinterpret_cast<uint32_t*>(p);
  p += align256(sizeof(uint32_t) * cap);
  m.hash = reinterpret_cast<uint64_t*>(p);
  p += align256(sizeof(uint64_t) * cap);
  m.key = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * NCFG * static_cast<size_t>(cap));
  m.bits = reinterpret_cast<uint32_t*>(p);
  p += align256(sizeof(uint32_t) * m.ws * static_cast<size_t>(cap));
  const size_t ncap = static_cast<size_t>(cap) * kNodesPerEntry;
  m.nodes.cap = static_cast<int32_t>(ncap);
  m.nodes.full = m.epoch + kHdrNodesFull;
  m.nodes.hash = reinterpret_cast<unsigned long long*>(p);
  p += align256(sizeof(unsigned long long) * ncap);
  m.nodes.ready = reinterpret_cast<uint32_t*>(p);
  p += align256(sizeof(uint32_t) * ncap);
  m.nodes.trans = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * 256 * ncap);
  m.nodes.key = reinterpret_cast<int32_t*>(p);
  return m;
}

// Bytes of the node table's parts that a reset zeroes (hash, ready, trans),
// counted from nodes.hash.
size_t nodes_clear_bytes(int32_t cap) {
  const size_t ncap = static_cast<size_t>(cap) * kNodesPerEntry;
  return align256(sizeof(unsigned long long) * ncap) + align256(sizeof(uint32_t) * ncap) +
         align256(sizeof(int32_t) * 256 * ncap);
}

// Bytes from nodes.hash that free every node slot (hash and ready words);
// a slot's transitions are reset by the warp that claims it.
size_t nodes_free_bytes(int32_t cap) {
  const size_t ncap = static_cast<size_t>(cap) * kNodesPerEntry;
  return align256(sizeof(unsigned long long) * ncap) + align256(sizeof(uint32_t) * ncap);
}

size_t memo_bytes(int32_t cap, int32_t vocab) {
  const size_t ncap = static_cast<size_t>(cap) * kNodesPerEntry;
  return 256 + align256(sizeof(uint32_t) * cap) + align256(sizeof(uint64_t) * cap) +
         align256(sizeof(int32_t) * NCFG * static_cast<size_t>(cap)) +
         align256(sizeof(uint32_t) * words_stride(vocab) * static_cast<size_t>(cap)) +
         nodes_clear_bytes(cap) + align256(sizeof(int32_t) * NCFG * ncap);
}

// Row kinds (Work::kind).
constexpr int32_t kBroken = 0, kHit = 1, kRep = 2, kAlias = 3;

struct Work {
  int32_t* dedup;    // [dcap] row index + 1 of the representative, 0 = empty
  int32_t dcap;      // power of two >= 2 * batch
  int32_t* counters; // [4] right after dedup (cleared with it): representatives,
                     //     next compute item, next first-byte item
  void* step;        // scratch of the fused step (cleared with dedup)
  size_t clear_bytes;  // bytes from dedup that every mask pipeline zeroes
  int32_t* reps;     // [batch] representative rows, in claim order
  int32_t* kind;     // [batch]
  int32_t* ref;      // [batch] memo entry (kHit, kRep with memo), rep row (kAlias), -1
  uint64_t* hash;    // [batch]
  uint32_t* first;   // [batch][8] surviving first bytes (representatives)
  int32_t* eos_ok;   // [batch]
  int32_t* node;     // [batch] node of a representative's config-set (-1: none)
  uint32_t* bits;    // [batch][ws] allow rows of representatives without a memo entry
};

constexpr int32_t pow2_at_least(int32_t x) {
  int32_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

Work work_view(void* base, int32_t batch, int32_t vocab) {
  Work w{};
  w.dcap = pow2_at_least(std::max(2 * batch, 2));
  char* p = static_cast<char*>(base);
  w.dedup = reinterpret_cast<int32_t*>(p);
  w.counters = w.dedup + w.dcap;
  p += align256(sizeof(int32_t) * (w.dcap + 4));
  w.step = p;
  p += step_scratch_bytes(batch);
  w.clear_bytes = static_cast<size_t>(p - static_cast<char*>(base));
  w.reps = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * batch);
  w.kind = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * batch);
  w.ref = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * batch);
  w.hash = reinterpret_cast<uint64_t*>(p);
  p += align256(sizeof(uint64_t) * batch);
  w.first = reinterpret_cast<uint32_t*>(p);
  p += align256(sizeof(uint32_t) * 8 * batch);
  w.eos_ok = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * batch);
  w.node = reinterpret_cast<int32_t*>(p);
  p += align256(sizeof(int32_t) * batch);
  w.bits = reinterpret_cast<uint32_t*>(p);
  return w;
}

constexpr size_t work_bytes(int32_t batch, int32_t vocab) {
  const int32_t dcap = pow2_at_least(2 * batch > 2 ? 2 * batch : 2);
  return align256(sizeof(int32_t) * (dcap + 4)) + step_scratch_bytes(batch) +
         3 * align256(sizeof(int32_t) * batch) +
         align256(sizeof(uint64_t) * batch) + align256(sizeof(uint32_t) * 8 * batch) +
         2 * align256(sizeof(int32_t) * batch) +
         align256(sizeof(uint32_t) * words_stride(vocab) * static_cast<size_t>(batch));
}

// murmur3's 64-bit finaliser (a published avalanche mix).
__device__ __forceinline__ uint64_t fmix64(uint64_t x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdULL;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ULL;
  x ^= x >> 33;
  return x;
}

// Word k of the canonical form of config-set c: the live content (number of
// configs, their depths and frames) with `saturated` and every word outside
// the live region zero. Memo keys are stored in this form, so two sets have
// the same mask key iff their canonical words are equal.
__device__ __forceinline__ int32_t canon_word(const int32_t* c, int k) {
  const int n = c[0];
  if (k == 0) return n;
  if (k == 1) return 0;
  if (k < 2 + MC) return (k - 2) < n ? c[k] : 0;
  const int i = (k - 2 - MC) / MD, f = (k - 2 - MC) % MD;
  return (i < n && f < c[2 + i]) ? c[k] : 0;
}

constexpr int kRowWords = (NCFG + 31) / 32;  // words of a config row per lane

// Warp-wide copy of a config row into shared memory: every load is issued
// before the first store (one memory round trip, 128-byte coalesced).
__device__ __forceinline__ void w_load_row(const int32_t* __restrict__ src, int32_t* dst,
                                           int lane) {
  int32_t v[kRowWords];
#pragma unroll
  for (int j = 0; j < kRowWords; ++j) {
    const int k = lane + 32 * j;
    v[j] = k < NCFG ? src[k] : 0;
  }
#pragma unroll
  for (int j = 0; j < kRowWords; ++j) {
    const int k = lane + 32 * j;
    if (k < NCFG) dst[k] = v[j];
  }
  __syncwarp();
}

// Hash of the canonical form (position-tagged words; config order matters,
// as it does for the mask under saturation).
__device__ uint64_t w_hash(const int32_t* c, int lane) {
  uint64_t h = 0;
#pragma unroll
  for (int j = 0; j < kRowWords; ++j) {
    const int k = lane + 32 * j;
    const int32_t v = k < NCFG ? canon_word(c, k) : 0;
    if (v != 0) h ^= fmix64((static_cast<uint64_t>(k + 1) << 32) ^ static_cast<uint32_t>(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) h ^= __shfl_xor_sync(kAll, h, o);
  return fmix64(h);
}

// Same live content: config-set `a` (shared memory) against canonical words
// held by each lane (key[j] = canonical word lane + 32 j of the other set).
__device__ __forceinline__ bool w_same_words(const int32_t* a, const int32_t (&key)[kRowWords],
                                             int lane) {
  bool eq = true;
#pragma unroll
  for (int j = 0; j < kRowWords; ++j) {
    const int k = lane + 32 * j;
    if (k < NCFG) eq &= canon_word(a, k) == key[j];
  }
  return __all_sync(kAll, eq);
}

__device__ __forceinline__ int64_t slot_of(const int64_t* slots, int32_t b) {
  return slots ? slots[b] : b;
}

// ---------------------------------------------------------------------------
// Transition cache (see Nodes). Waits are bounded: a warp that finds a slot
// or a transition another warp is filling polls it at most kNodePolls times
// (the filler is a running warp that waits on nothing itself) and then goes
// on without it -- a duplicate node or a recomputed transition, never a
// different result.

constexpr int kNodeProbe = 64;
constexpr int kNodePolls = 1 << 14;
constexpr int32_t kTransUnknown = 0, kTransBusy = 1, kTransDead = 2, kTransNode = 3;

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int32_t ld_acquire_s32(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Node of config-set `c` (shared memory; any words outside its live region)
// with content hash `h`: found, or claimed and written here; -1 when the
// probe sequence is full.
__device__ int32_t node_intern(const Nodes& nd, const int32_t* c, uint64_t h, int lane) {
  const unsigned long long hv = static_cast<unsigned long long>(h) | 1ull;
  for (int p = 0; p < kNodeProbe; ++p) {
    const int32_t e = static_cast<int32_t>((h + static_cast<uint64_t>(p)) &
                                           static_cast<uint64_t>(nd.cap - 1));
    unsigned long long cur = 0;
    if (lane == 0) {
      cur = atomicAdd(nd.hash + e, 0ull);
      if (cur == 0ull) cur = atomicCAS(nd.hash + e, 0ull, hv);
    }
    cur = __shfl_sync(kAll, cur, 0);
    if (cur == 0ull) {  // this warp claimed the slot: write the key, then publish it
      // the slot may have held a node before the table was started over (only
      // its hash and ready words are cleared then): no transition is known yet
      int32_t* tr = nd.trans + static_cast<int64_t>(e) * 256;
      for (int k = lane; k < 256; k += 32) tr[k] = kTransUnknown;
      int32_t* key = nd.key + static_cast<int64_t>(e) * NCFG;
      for (int k = lane; k < NCFG; k += 32) key[k] = canon_word(c, k);
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicExch(nd.ready + e, 1u);
      return e;
    }
    if (cur != hv) continue;
    uint32_t rdy = 0;
    if (lane == 0) {
      rdy = ld_acquire_u32(nd.ready + e);
      for (int i = 0; rdy == 0u && i < kNodePolls; ++i) {
        __nanosleep(64);
        rdy = ld_acquire_u32(nd.ready + e);
      }
    }
    rdy = __shfl_sync(kAll, rdy, 0);
    if (rdy == 0u) continue;  // not written in time: look further (a duplicate at worst)
    __syncwarp();
    const int32_t* key = nd.key + static_cast<int64_t>(e) * NCFG;
    int32_t kw[kRowWords];
#pragma unroll
    for (int j = 0; j < kRowWords; ++j) {
      const int k = lane + 32 * j;
      kw[j] = k < NCFG ? __ldcg(key + k) : 0;
    }
    if (w_same_words(c, kw, lane)) return e;
  }
  if (lane == 0) atomicOr(nd.full, 1u);  // the next call starts on an empty table
  return -1;
}

// The node after byte `byte` from node q: >= 0 a node, -1 the set dies, -2
// the next set could not be interned (table full) -- then `next` holds it.
// `cur` and `next` are NCFG words of this warp's shared memory. A known
// transition is read from the table; an unknown one is computed here (the
// bounded closure, w_advance_byte, on q's content) and stored.
__device__ int32_t node_step(const bpd_pda_grammar& g, const Nodes& nd, int32_t q, int byte,
                             int32_t* cur, int32_t* next, int lane, bool key_ready = false) {
  if (q < 0 || q >= nd.cap) return -2;  // not a node: callers never pass one
  int32_t* slot = nd.trans + static_cast<int64_t>(q) * 256 + byte;
  int32_t v = 0;
  bool own = false;
  if (lane == 0) {
    v = ld_acquire_s32(slot);
    if (v == kTransUnknown) {
      v = atomicCAS(slot, kTransUnknown, kTransBusy);
      own = v == kTransUnknown;
    }
    for (int i = 0; v == kTransBusy && !own && i < kNodePolls; ++i) {
      __nanosleep(64);
      v = ld_acquire_s32(slot);
    }
  }
  own = __shfl_sync(kAll, own, 0);
  v = __shfl_sync(kAll, v, 0);
  if (!own && v == kTransDead) return -1;
  if (!own && v >= kTransNode && v - kTransNode < nd.cap) return v - kTransNode;
  // compute it (owner, or after a wait that ran out: then without storing);
  // q came from a transition another warp may have stored just now: order
  // the key's reads after it (unless the caller already holds q's key in cur)
  if (!key_ready) {
    __threadfence();
    const int32_t* key = nd.key + static_cast<int64_t>(q) * NCFG;
    for (int k = lane; k < NCFG; k += 32) cur[k] = __ldcg(key + k);
    __syncwarp();
  }
  int32_t r = -1;
  if (w_advance_byte<false>(g, cur, next, byte, lane)) {
    const int32_t e = node_intern(nd, next, w_hash(next, lane), lane);
    r = e >= 0 ? e : -2;
  }
  if (own && lane == 0) {
    __threadfence();
    atomicExch(slot, r == -1 ? kTransDead : r >= 0 ? kTransNode + r : kTransUnknown);
  }
  return r;
}

// ---------------------------------------------------------------------------
// Mask pipeline.

// One warp per row, its config-set copied once into shared memory `A` (`B`:
// scratch for a dedup comparison): memo lookup and in-batch dedup. A row
// whose content is neither in the memo nor already claimed by an equal row of
// this call becomes a representative: it is appended to the representative
// list and its first-byte table is cleared for the first-byte phase.
__device__ __forceinline__ void lookup_row(const bpd_pda_grammar& g,
                                           const int32_t* __restrict__ pool,
                                           const int64_t* __restrict__ slots,
                                           const uint8_t* __restrict__ broken, int32_t b,
                                           const Memo& memo, const Work& w, int32_t* A,
                                           int32_t* B) {
  const int lane = threadIdx.x & 31;
  const int64_t slot = slot_of(slots, b);
  // this call's tag, loaded beside the row (it does not depend on it)
  const uint32_t epoch = memo.cap ? *memo.epoch : 0u;
  const bool brk = broken != nullptr && broken[slot] != 0;
  w_load_row(pool + slot * NCFG, A, lane);
  if (brk) {
    if (lane == 0) {
      w.kind[b] = kBroken;
      w.ref[b] = -1;
    }
    return;
  }
  const uint64_t h = w_hash(A, lane);
  int32_t kind = kRep, ref = -1;
  uint32_t cur = 0;  // this call's tag
  if (memo.cap) {
    cur = epoch + 1u;
    if (cur == 0u) cur = 1u;
  }
  // memo: entries claimed earlier in this call (tag == cur) are still being
  // filled and are skipped; equal content claimed by this call is found
  // through the in-batch dedup below instead. An entry's tag, hash and key
  // words are loaded together (one round trip per probe).
  for (int p = 0; memo.cap && p < kProbe; ++p) {
    const int32_t e = static_cast<int32_t>((h + p) & (memo.cap - 1));
    const int32_t* key = memo.key + static_cast<int64_t>(e) * NCFG;
    const uint32_t tag = memo.tag[e];
    const uint64_t eh = memo.hash[e];
    int32_t kw[kRowWords];
#pragma unroll
    for (int j = 0; j < kRowWords; ++j) {
      const int k = lane + 32 * j;
      kw[j] = k < NCFG ? key[k] : 0;
    }
    if (tag == 0u) break;
    if (tag == cur) continue;
    if (eh == h && w_same_words(A, kw, lane)) {
      kind = kHit;
      ref = e;
      break;
    }
  }
  if (kind != kHit) {
    // in-batch dedup: the first row to claim a dedup slot for this content is
    // the representative; equal rows become its aliases (compared on the
    // other row's pool content, which this call never writes)
    for (int p = 0; p < w.dcap; ++p) {
      const int32_t d = static_cast<int32_t>((h + p) & (w.dcap - 1));
      int32_t prev = 0;
      if (lane == 0) prev = atomicCAS(w.dedup + d, 0, b + 1);
      prev = __shfl_sync(kAll, prev, 0);
      if (prev == 0) break;  // representative
      const int32_t other = prev - 1;
      w_load_row(pool + slot_of(slots, other) * NCFG, B, lane);
      int32_t ow[kRowWords];
#pragma unroll
      for (int j = 0; j < kRowWords; ++j) {
        const int k = lane + 32 * j;
        ow[j] = k < NCFG ? canon_word(B, k) : 0;
      }
      if (w_same_words(A, ow, lane)) {
        kind = kAlias;
        ref = other;
        break;
      }
    }
  }
  if (kind == kRep) {
    if (lane < 8) w.first[static_cast<int64_t>(b) * 8 + lane] = 0u;
    if (lane == 0) {
      w.reps[atomicAdd(w.counters + 0, 1)] = b;
      w.eos_ok[b] = is_complete(g, A) ? 1 : 0;
    }
    // claim a memo entry (none free along the probe: bits go to the workspace)
    for (int p = 0; memo.cap && p < kProbe; ++p) {
      const int32_t e = static_cast<int32_t>((h + p) & (memo.cap - 1));
      uint32_t prev = 0;
      if (lane == 0) prev = atomicCAS(memo.tag + e, 0u, cur);
      prev = __shfl_sync(kAll, prev, 0);
      if (prev == 0u) {
        int32_t* key = memo.key + static_cast<int64_t>(e) * NCFG;
        for (int k = lane; k < NCFG; k += 32) key[k] = canon_word(A, k);
        if (lane == 0) memo.hash[e] = h;
        ref = e;
        break;
      }
    }
  }
  if (kind == kRep) {
    // the representative's node: its walks start there
    const int32_t nd = (BPD_PDA_NODES && memo.nodes.cap) ? node_intern(memo.nodes, A, h, lane)
                                                         : -1;
    if (lane == 0) w.node[b] = nd;
  }
  if (lane == 0) {
    w.kind[b] = kind;
    w.ref[b] = ref;
    w.hash[b] = h;
  }
}

// Which first bytes keep each representative's set alive: one warp per
// (representative, byte) item, items taken from a counter so the whole grid
// works on however many representatives this call has (none: every warp
// exits at once).
__device__ __forceinline__ void first_byte_items(const bpd_pda_grammar& g,
                                                 const int32_t* __restrict__ pool,
                                                 const int64_t* __restrict__ slots,
                                                 const Work& w, int32_t* scratch) {
  const int lane = threadIdx.x & 31;
  const int32_t items = w.counters[0] * 256;
  if (items == 0) return;  // every row hit the memo: no item, no atomics
  for (;;) {
    int32_t item = 0;
    if (lane == 0) item = atomicAdd(w.counters + 2, 1);
    item = __shfl_sync(kAll, item, 0);
    if (item >= items) break;
    const int32_t b = w.reps[item >> 8];
    const int byte = item & 255;
    const int32_t* base = pool + slot_of(slots, b) * NCFG;
    const bool ok = w_advance_byte<false>(g, base, scratch, byte, lane);
    if (ok && lane == 0) atomicOr(w.first + static_cast<int64_t>(b) * 8 + (byte >> 5), 1u << (byte & 31));
  }
}

__device__ __forceinline__ uint32_t* rep_bits(const Memo& memo, const Work& w, int32_t b) {
  const int32_t e = w.ref[b];
  if (memo.cap && e >= 0) return memo.bits + static_cast<int64_t>(e) * memo.ws;
  return w.bits + static_cast<int64_t>(b) * memo.ws;
}

// Token walks of a warp through the transition cache, lane = token: a lane
// with `walk` set follows its token's bytes from node nd0, from the first
// byte on. Transitions the table does not hold yet are computed by the
// whole warp, one at a time (node_step; another warp computing the same one
// is waited for, boundedly); a lane whose next set cannot be interned
// finishes its token with direct byte steps from that set. Sets `ok` of
// every lane with `walk`.
__device__ __forceinline__ void node_walk(const bpd_pda_grammar& g, const Nodes& nd, int32_t nd0,
                                          int32_t o0, int32_t o1, bool walk, bool& ok,
                                          int32_t (*buf)[NCFG], int lane) {
  bool active = walk;
  int32_t q = nd0, i = o0;
  for (;;) {
    int32_t byte = 0;
    while (active) {
      if (i == o1) {
        ok = true;
        active = false;
        break;
      }
      byte = __ldg(g.tok_bytes + i);
      const int32_t v = __ldcg(nd.trans + static_cast<int64_t>(q) * 256 + byte);
      if (v >= kTransNode && v - kTransNode < nd.cap) {
        q = v - kTransNode;
        ++i;
      } else if (v == kTransDead) {
        ok = false;
        active = false;
      } else {
        break;  // unknown, or being computed: the warp takes it below
      }
    }
    const uint32_t need = __ballot_sync(kAll, active);
    if (need == 0u) break;
    const int j = __ffs(need) - 1;
    const int32_t qj = __shfl_sync(kAll, q, j);
    const int32_t bj = __shfl_sync(kAll, byte, j);
    const int32_t r = node_step(g, nd, qj, bj, buf[0], buf[1], lane);
    if (r == -2) {
      // not interned: the rest of lane j's token by direct byte steps
      const int32_t k0 = __shfl_sync(kAll, i, j) + 1, k1 = __shfl_sync(kAll, o1, j);
      const int32_t* c = buf[1];
      bool alive = true;
      for (int32_t k = k0; k < k1 && alive; ++k) {
        int32_t* n = c == buf[1] ? buf[0] : buf[1];
        alive = w_advance_byte<false>(g, c, n, __ldg(g.tok_bytes + k), lane);
        c = n;
      }
      if (lane == j) {
        ok = alive;
        active = false;
      }
    } else if (lane == j) {
      if (r == -1) {
        ok = false;
        active = false;
      } else {
        q = r;
        ++i;
      }
    }
  }
}

constexpr int32_t kComputeChunk = kWarps * 32 * 4;  // tokens per compute item
constexpr int32_t kPrefillItems = 256 / (kWarps * 4);  // first-byte items per node (4 bytes a warp)

// Allow bits of every representative row. Items are taken from a counter by a
// resident grid: first, per representative with a node, kPrefillItems items
// that fill the node's 256 first-byte transitions (4 bytes a warp, each one
// bounded closure unless already known), so a new node's first steps are
// computed in parallel; then (representative, 1024 tokens) items, each warp
// deciding 32 tokens at a time (lane = token). With a node, the item's copy of
// the node's first-byte row in shared memory rejects a token whose first byte
// kills the set with one shared read and starts a longer token's walk at the
// node after its first byte; transitions not known when the row was copied
// go through the table (node_walk). Without a node, only tokens whose first
// byte survives (first_byte_kernel) and that are longer than one byte are
// walked directly.
__device__ __forceinline__ void compute_items(const bpd_pda_grammar& g,
                                              const int32_t* __restrict__ pool,
                                              const int64_t* __restrict__ slots,
                                              const Memo& memo, const Work& w,
                                              bool first_valid, int32_t (*buf)[2][NCFG],
                                              uint32_t* first, int32_t* strans,
                                              int32_t& s_item) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int32_t V = g.vocab_size;
  const int32_t chunks = (V + kComputeChunk - 1) / kComputeChunk;
  const int32_t reps = w.counters[0];
  const bool nodes = memo.nodes.cap > 0 && !first_valid;
  const int32_t prefill = nodes ? reps * kPrefillItems : 0;
  const int32_t items = prefill + reps * chunks;
  if (items == 0) return;  // the same value for every thread of the CTA
  for (;;) {
    __syncthreads();  // the previous item's shared state is no longer read
    if (threadIdx.x == 0) s_item = atomicAdd(w.counters + 1, 1);
    __syncthreads();
    const int32_t item = s_item;
    if (item >= items) break;
    if (item < prefill) {
      // first-byte transitions of a representative's node, 4 bytes a warp
      const int32_t nd = w.node[w.reps[item / kPrefillItems]];
      if (nd >= 0) {
        // the node's key once for the warp's 4 bytes (the node was interned by
        // the lookup kernel, which has completed; node_step leaves cur intact)
        int32_t* cur = buf[warp][0];
        const int32_t* key = memo.nodes.key + static_cast<int64_t>(nd) * NCFG;
        for (int k = lane; k < NCFG; k += 32) cur[k] = __ldcg(key + k);
        __syncwarp();
        const int32_t b0 = (item % kPrefillItems) * (kWarps * 4) + warp * 4;
        for (int k = 0; k < 4; ++k)
          node_step(g, memo.nodes, nd, b0 + k, cur, buf[warp][1], lane, true);
      }
      continue;
    }
    const int32_t ti = item - prefill;
    const int32_t b = w.reps[ti / chunks];
    const int32_t c0 = (ti % chunks) * kComputeChunk;
    const int32_t c1 = min(V, c0 + kComputeChunk);
    const int32_t* base = pool + slot_of(slots, b) * NCFG;
    const int32_t nd0 = w.node[b];
    if (first_valid && threadIdx.x < 8)
      first[threadIdx.x] = w.first[static_cast<int64_t>(b) * 8 + threadIdx.x];
    if (nd0 >= 0) {
      for (int k = threadIdx.x; k < 256; k += blockDim.x)
        strans[k] = __ldcg(memo.nodes.trans + static_cast<int64_t>(nd0) * 256 + k);
    }
    __syncthreads();
    const bool eos_ok = w.eos_ok[b] != 0;
    const bool nonempty = n_of(base) > 0;
    uint32_t* out = rep_bits(memo, w, b);
    // each lane's token offsets are loaded one iteration ahead
    int32_t n_o0 = 0, n_o1 = 0;
    if (c0 + warp * 32 + lane < c1) {
      n_o0 = __ldg(g.tok_offsets + c0 + warp * 32 + lane);
      n_o1 = __ldg(g.tok_offsets + c0 + warp * 32 + lane + 1);
    }
    for (int32_t t0 = c0 + warp * 32; t0 < c1; t0 += kWarps * 32) {
      const int32_t t = t0 + lane;
      bool ok = false, walk = false;
      int32_t o0 = n_o0, o1 = n_o1;
      if (t + kWarps * 32 < c1) {
        n_o0 = __ldg(g.tok_offsets + t + kWarps * 32);
        n_o1 = __ldg(g.tok_offsets + t + kWarps * 32 + 1);
      }
      int32_t q = nd0;  // the node a lane's walk starts from (with a node)
      if (t >= c1) {
        o0 = o1 = 0;
      } else {
        if (t == g.eos_id) {
          ok = eos_ok;
          o0 = o1 = 0;
        } else {
          if (o0 == o1) {
            ok = nonempty;
          } else if (nd0 >= 0) {
            // the first byte through the node's row copied above
            const int32_t v = strans[__ldg(g.tok_bytes + o0)];
            if (v == kTransDead) {
              // the set dies on the first byte: rejected
            } else if (v >= kTransNode && v - kTransNode < memo.nodes.cap) {
              if (o1 - o0 == 1) {
                ok = true;
              } else {
                q = v - kTransNode;
                ++o0;
                walk = true;
              }
            } else {
              walk = true;  // not known when copied: through the table
            }
          } else if (!first_valid) {
            walk = true;  // a direct walk
          } else {
            const int fb = __ldg(g.tok_bytes + o0);
            if ((first[fb >> 5] >> (fb & 31)) & 1u) {
              if (o1 - o0 == 1) ok = true;
              else walk = true;
            }
          }
        }
      }
      if (nd0 >= 0) {
        node_walk(g, memo.nodes, q, o0, o1, walk, ok, buf[warp], lane);
        walk = false;
      }
      uint32_t todo = __ballot_sync(kAll, walk);
      while (todo) {
        const int j = __ffs(todo) - 1;
        todo &= todo - 1;
        const int32_t s = __shfl_sync(kAll, o0, j);
        const int32_t e = __shfl_sync(kAll, o1, j);
        const int32_t* cur = base;
        int which = 0;
        bool alive = true;
        for (int32_t i = s; i < e && alive; ++i) {
          int32_t* nxt = buf[warp][which];
          alive = w_advance_byte<false>(g, cur, nxt, __ldg(g.tok_bytes + i), lane);
          cur = nxt;
          which ^= 1;
        }
        if (lane == j) ok = alive;
      }
      const uint32_t word = __ballot_sync(kAll, ok);
      if (lane == 0) out[t0 >> 5] = word;
    }
  }
}

constexpr int kLookupWarps = 4;

// The mask pipeline's kernels, in stream order after prologue_kernel clears
// the call's dedup table and counters: memo lookup and in-batch dedup (a warp
// per row), first bytes of the representatives (without a memo only), their
// allow bits. With every row a memo hit the last two find no items and end
// at once.
__global__ void __launch_bounds__(kLookupWarps * 32)
    lookup_kernel(bpd_pda_grammar g, const int32_t* __restrict__ pool,
                  const int64_t* __restrict__ slots, const uint8_t* __restrict__ broken,
                  int32_t batch, Memo memo, Work w, const int32_t* __restrict__ nrows) {
  __shared__ int32_t buf[kLookupWarps][2][NCFG];
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5;
  const int32_t b = blockIdx.x * kLookupWarps + warp;
  const int32_t n = nrows != nullptr ? min(batch, *nrows) : batch;
  if (b < n) lookup_row(g, pool, slots, broken, b, memo, w, buf[warp][0], buf[warp][1]);
}

__global__ void __launch_bounds__(kThreads)
    first_byte_kernel(bpd_pda_grammar g, const int32_t* __restrict__ pool,
                      const int64_t* __restrict__ slots, Work w) {
  __shared__ int32_t scratch[kWarps][NCFG];
  pdl_trigger();
  pdl_wait();
  first_byte_items(g, pool, slots, w, scratch[threadIdx.x >> 5]);
}

__global__ void __launch_bounds__(kThreads)
    compute_kernel(bpd_pda_grammar g, const int32_t* __restrict__ pool,
                   const int64_t* __restrict__ slots, Memo memo, Work w, int32_t first_valid) {
  __shared__ int32_t buf[kWarps][2][NCFG];
  __shared__ uint32_t first[8];
  __shared__ int32_t strans[256];
  __shared__ int32_t s_item;
  pdl_trigger();
  pdl_wait();
  compute_items(g, pool, slots, memo, w, first_valid != 0, buf, first, strans, s_item);
  // the last kernel of every mask call: the next call gets a new tag (the
  // lookups of this call, which read the old epoch, have all finished)
  if (memo.cap && blockIdx.x == 0 && threadIdx.x == 0) {
    uint32_t cur = *memo.epoch + 1u;
    if (cur == 0u) cur = 1u;
    *memo.epoch = cur;
  }
}

__device__ __forceinline__ const uint32_t* row_bits(const Memo& memo, const Work& w, int32_t b) {
  const int32_t kind = w.kind[b];
  if (kind == kBroken) return nullptr;
  if (kind == kHit) return memo.bits + static_cast<int64_t>(w.ref[b]) * memo.ws;
  const int32_t rep = kind == kAlias ? w.ref[b] : b;
  return rep_bits(memo, w, rep);
}

// Row -> its allow words through the memo / workspace (nullptr for broken rows).
// PDA rows are mostly rejected tiles (bulk fills in place, nothing read from
// the model's rows): a CTA takes twice the dense chunk (8 warp tiles a warp),
// so fewer CTAs per row meet in the argmax merge and fewer blocks of a step
// over a device-held row count find no row. Config 4 (256 rows, in place):
// 39.0 against 40.1-40.8 us per step from a graph, the miss-path workloads
// unchanged; the config-5 serving step, whose PDA rows run beside the dense
// rows' step: 127.4 against 133.5 us (same box).
#ifndef BPD_PDA_TILES_PER_WARP
#define BPD_PDA_TILES_PER_WARP 8
#endif

struct PdaRows {
  static constexpr bool kSoft = false;
  static constexpr int kTilesPerWarp = BPD_PDA_TILES_PER_WARP;
  Memo memo;
  Work w;
  __device__ __forceinline__ RowInfo operator()(int32_t row) const {
    return RowInfo{row_bits(memo, w, row), 0, 0};
  }
};

// Advance config-set pool[slots[b]] by token t, one warp, with 3 * NCFG
// int32 of shared memory: an exact trial walk of the token's bytes, written
// back only if every byte is accepted; EOS never changes the config-set and
// is accepted iff it is complete (pda_cpu.cpp:35-54). Then ok / broken /
// status as grammar/device.py:268-283.
__device__ __forceinline__ void warp_commit_token(const bpd_pda_grammar& g, int32_t* pool,
                                                  int64_t slot, int32_t b, int64_t t,
                                                  int32_t* buf, uint8_t* ok_out, uint8_t* broken,
                                                  int32_t* status_out) {
  const int lane = threadIdx.x & 31;
  int32_t* row = pool + slot * NCFG;
  int32_t* trial = buf;
  w_copy(trial, row, lane);
  bool ok;
  if (t == g.eos_id) {
    ok = is_complete(g, trial);  // EOS never changes the config-set
  } else if (t < 0 || t >= g.vocab_size) {
    ok = false;
  } else {
    const int32_t s = __ldg(g.tok_offsets + t), e = __ldg(g.tok_offsets + t + 1);
    const int32_t* cur = trial;
    int which = 1;
    ok = true;
    for (int32_t i = s; i < e && ok; ++i) {
      int32_t* nxt = buf + which * NCFG;
      ok = w_advance_byte<true>(g, cur, nxt, __ldg(g.tok_bytes + i), lane);
      cur = nxt;
      which = which == 1 ? 2 : 1;
    }
    if (ok && cur != trial) {
      for (int k = lane; k < NCFG; k += 32) row[k] = cur[k];
    }
  }
  if (lane == 0) {
    if (ok_out) ok_out[b] = ok ? 1 : 0;
    if (broken) {
      const uint8_t br = static_cast<uint8_t>(broken[slot] | (ok ? 0 : 1));
      broken[slot] = br;
      if (status_out) status_out[b] = br ? -1 : 1;
    } else if (status_out) {
      status_out[b] = ok ? 1 : -1;
    }
  }
}

// Commit of the fused PDA step: record the token and advance the row's
// config-set by it, in the warp that finished the row.
struct PdaCommit {
  static constexpr int kSmemBytes = 3 * NCFG * static_cast<int>(sizeof(int32_t));
  bpd_pda_grammar g;
  int32_t* pool;
  const int64_t* slots;
  int64_t* token_out;
  uint8_t* broken;
  int32_t* status_out;
  __device__ __forceinline__ void operator()(int32_t row, const RowInfo&, int32_t tok,
                                             uint8_t* smem) const {
    if ((threadIdx.x & 31) == 0) token_out[row] = tok;
    warp_commit_token(g, pool, slot_of(slots, row), row, tok, reinterpret_cast<int32_t*>(smem),
                      nullptr, broken, status_out);
  }
};

__global__ void pda_bits_out_kernel(int32_t W, Memo memo, Work w, uint32_t* __restrict__ out) {
  const int32_t row = blockIdx.y;
  const uint32_t* src = row_bits(memo, w, row);
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < W; i += gridDim.x * blockDim.x)
    out[static_cast<int64_t>(row) * W + i] = src ? src[i] : 0u;
}

// ---------------------------------------------------------------------------
// Commit, init, completeness.

constexpr int kAdvWarps = 4;

// One warp per row: the exact byte walk of pda_cpu.cpp:35-54 in shared memory;
// the final config-set is written back only if the token was accepted.
__global__ void __launch_bounds__(kAdvWarps * 32)
    advance_kernel(bpd_pda_grammar g, int32_t* __restrict__ pool, const int64_t* __restrict__ slots,
                   int32_t batch, const void* __restrict__ tokens, int32_t tokens64,
                   uint8_t* __restrict__ ok_out, uint8_t* __restrict__ broken,
                   int32_t* __restrict__ status_out) {
  __shared__ int32_t buf[kAdvWarps][3 * NCFG];
  const int warp = threadIdx.x >> 5;
  const int32_t b = blockIdx.x * kAdvWarps + warp;
  if (b >= batch) return;
  const int64_t t = tokens64 ? static_cast<const int64_t*>(tokens)[b]
                             : static_cast<int64_t>(static_cast<const int32_t*>(tokens)[b]);
  warp_commit_token(g, pool, slot_of(slots, b), b, t, buf[warp], ok_out, broken, status_out);
}

// pda.hpp:200-207 on a zeroed struct (as the reference's pda_init op).
__global__ void init_kernel(bpd_pda_grammar g, int32_t* __restrict__ out) {
  __shared__ int32_t c[NCFG];
  const int lane = threadIdx.x;
  for (int k = lane; k < NCFG; k += 32) c[k] = 0;
  __syncwarp();
  w_push(c, 1, lane == 0 ? g.root_start : 0, lane);
  w_close(g, c, lane);
  for (int k = lane; k < NCFG; k += 32) out[k] = c[k];
}

__global__ void complete_kernel(bpd_pda_grammar g, const int32_t* __restrict__ pool,
                                const int64_t* __restrict__ slots,
                                const uint8_t* __restrict__ broken, int32_t batch,
                                uint8_t* __restrict__ out) {
  const int32_t b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const int64_t slot = slot_of(slots, b);
  out[b] = (!(broken && broken[slot]) && is_complete(g, pool + slot * NCFG)) ? 1 : 0;
}

// The first launch of every mask call, in place of a memset: zero the call's
// dedup table, counters and step scratch (Work::clear_bytes from w.dedup)
// and, when the previous call found the transition cache full (a node it
// could not intern), every node slot's hash and ready words (768 KB at the
// default capacity; a claimed slot's transitions are reset by the warp that
// claims it, and no walk reaches a node of the old table: walks start at
// nodes of the running call and follow transitions stored since the table
// started over) -- so a grammar whose walks keep
// reaching new config-sets starts each call with room instead of falling
// back to direct walks for good. Every CTA reads the flag before it counts
// itself done, and the last CTA out clears flag and count, so all CTAs act
// on the same flag value (when the flag is unset no CTA counts).
constexpr int kPrologueThreads = 256;

__global__ void __launch_bounds__(kPrologueThreads)
    prologue_kernel(Memo memo, Work w, size_t node_bytes) {
  pdl_trigger();
  pdl_wait();  // the previous call's kernels may still use this workspace
  const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
  uint4* wz = reinterpret_cast<uint4*>(w.dedup);
  for (size_t i = tid; i < w.clear_bytes / 16; i += stride) wz[i] = zero;
  if (memo.cap == 0 || node_bytes == 0) return;
  // nothing writes the flag while the prologue runs, so every thread of the
  // grid reads the same value: unset (the usual case), nothing more to do
  const uint32_t full = *reinterpret_cast<volatile uint32_t*>(memo.epoch + kHdrNodesFull);
  if (full == 0u) return;
  uint4* nz = reinterpret_cast<uint4*>(memo.nodes.hash);
  for (size_t i = tid; i < node_bytes / 16; i += stride) nz[i] = zero;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t done;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(done)
                 : "l"(memo.epoch + kHdrPrologueDone)
                 : "memory");
    if (done == gridDim.x - 1u) {
      memo.epoch[kHdrNodesFull] = 0u;
      memo.epoch[kHdrPrologueDone] = 0u;
    }
  }
}

constexpr int kPrologueBlocks = 16;

bpd_status check_grammar(const bpd_pda_grammar* g) {
  BPD_REQUIRE(g != nullptr, "null grammar");
  BPD_REQUIRE(g->accept && g->live && g->edge_offsets && g->tok_offsets && g->tok_bytes,
              "grammar: null table pointer");
  BPD_REQUIRE(g->num_edges == 0 || (g->edge_kind && g->edge_lo && g->edge_hi && g->edge_dst &&
                                    g->edge_callee),
              "grammar: null edge pointer");
  BPD_REQUIRE(g->num_states > 0 && g->vocab_size > 0, "grammar: bad sizes");
  BPD_REQUIRE(g->root_start >= 0 && g->root_start < g->num_states, "grammar: bad root_start");
  return BPD_OK;
}

// prologue + lookup + claim + compute: leaves every row's allow bits
// resolvable through (memo, work).
bpd_status run_mask_pipeline(const bpd_pda_grammar* g, const int32_t* pool, const int64_t* slots,
                             const uint8_t* broken, int32_t batch, void* memo_mem, int32_t cap,
                             void* workspace, Memo* memo_out, Work* work_out, cudaStream_t st,
                             const int32_t* nrows = nullptr) {
  bpd_status rc = check_grammar(g);
  if (rc) return rc;
  BPD_REQUIRE(pool && workspace, "null config pool or workspace");
  BPD_REQUIRE(memo_mem == nullptr || (cap > 0 && (cap & (cap - 1)) == 0),
              "memo capacity must be a power of two");
  BPD_REQUIRE(aligned16(workspace) && (memo_mem == nullptr || aligned16(memo_mem)),
              "workspace and memo must be 16-byte aligned");
  Memo memo = memo_view(memo_mem, cap, g->vocab_size);
  Work w = work_view(workspace, batch, g->vocab_size);
  const int32_t sms = sm_count();
  const size_t node_bytes = (BPD_PDA_NODES && memo.nodes.cap > 0) ? nodes_free_bytes(cap) : 0;
  cudaError_t e = launch_pdl(prologue_kernel, dim3(kPrologueBlocks), dim3(kPrologueThreads), 0, st,
                             memo, w, node_bytes);
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "pda prologue_kernel: %s", cudaGetErrorString(e));
  rc = check_launch("pda prologue_kernel");
  if (rc) return rc;
  e = launch_pdl(lookup_kernel, dim3((batch + kLookupWarps - 1) / kLookupWarps),
                 dim3(kLookupWarps * 32), 0, st, *g, pool, slots, broken, batch, memo, w, nrows);
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "pda lookup_kernel: %s", cudaGetErrorString(e));
  rc = check_launch("pda lookup_kernel");
  if (rc) return rc;
  // With a transition cache the compute walks take every token from its
  // first byte through the cache; without one, the first bytes that keep
  // each representative alive are found first, so that tokens starting with
  // any other byte are rejected without a walk.
  const bool nodes = BPD_PDA_NODES && memo.nodes.cap > 0;
  if (!nodes) {
    e = launch_pdl(first_byte_kernel, dim3(sms * 2), dim3(kThreads), 0, st, *g, pool, slots, w);
    if (e != cudaSuccess)
      return fail(BPD_ERR_CUDA, "pda first_byte_kernel: %s", cudaGetErrorString(e));
    rc = check_launch("pda first_byte_kernel");
    if (rc) return rc;
  }
  e = launch_pdl(compute_kernel, dim3(sms * 2), dim3(kThreads), 0, st, *g, pool, slots, memo, w,
                 nodes ? 0 : 1);
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "pda compute_kernel: %s", cudaGetErrorString(e));
  rc = check_launch("pda compute_kernel");
  if (rc) return rc;
  *memo_out = memo;
  *work_out = w;
  return BPD_OK;
}

template <typename T>
bpd_status launch_pda_apply(void* logits, int64_t row_stride, int32_t batch, int32_t V,
                            const Memo& memo, const Work& w, float neg_inf, cudaStream_t st) {
  return launch_stream_apply<T, PdaRows>(logits, row_stride, batch, V, PdaRows{memo, w}, neg_inf,
                                         st, "pda apply kernel");
}

template <typename T>
bpd_status launch_pda_step(void* logits, int64_t row_stride, int32_t batch, int32_t V,
                           const Memo& memo, const Work& w, float neg_inf,
                           const PdaCommit& commit, int32_t chunks_per_row, cudaStream_t st) {
  return launch_stream_step<T, PdaRows, PdaCommit>(logits, row_stride, batch, V, PdaRows{memo, w},
                                                   commit, neg_inf, chunks_per_row, w.step, st,
                                                  "pda step kernel");
}

}  // namespace
}  // namespace bpd

using namespace bpd;

extern "C" bpd_status bpd_pda_init(const bpd_pda_grammar* g, int32_t* config_out, void* stream) {
  bpd_status rc = check_grammar(g);
  if (rc) return rc;
  BPD_REQUIRE(config_out != nullptr, "bpd_pda_init: null output");
  init_kernel<<<1, 32, 0, as_stream(stream)>>>(*g, config_out);
  return check_launch("pda init_kernel");
}

extern "C" size_t bpd_pda_memo_bytes(int32_t capacity, int32_t vocab_size) {
  if (capacity <= 0 || vocab_size <= 0) return 0;
  return memo_bytes(capacity, vocab_size);
}

extern "C" bpd_status bpd_pda_memo_reset(void* memo, int32_t capacity, int32_t vocab_size,
                                         void* stream) {
  BPD_REQUIRE(memo != nullptr, "bpd_pda_memo_reset: null memo");
  BPD_REQUIRE(capacity > 0 && (capacity & (capacity - 1)) == 0,
              "bpd_pda_memo_reset: capacity must be a power of two");
  BPD_REQUIRE(vocab_size > 0, "bpd_pda_memo_reset: bad vocab");
  Memo m = memo_view(memo, capacity, vocab_size);
  cudaError_t e = cudaMemsetAsync(m.epoch, 0, 256 + sizeof(uint32_t) * capacity,
                                  as_stream(stream));
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "memo reset: %s", cudaGetErrorString(e));
  e = cudaMemsetAsync(m.nodes.hash, 0, nodes_clear_bytes(capacity), as_stream(stream));
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "memo reset: %s", cudaGetErrorString(e));
  return BPD_OK;
}

extern "C" size_t bpd_pda_workspace_bytes(int32_t batch, int32_t vocab_size) {
  if (batch <= 0 || vocab_size <= 0) return 256;
  return work_bytes(batch, vocab_size);
}

extern "C" bpd_status bpd_pda_mask_bits(const bpd_pda_grammar* g, const int32_t* config_pool,
                                        const int64_t* slots, const uint8_t* broken,
                                        int32_t batch, void* memo, int32_t memo_capacity,
                                        void* workspace, uint32_t* out_bits, void* stream) {
  BPD_REQUIRE(batch >= 0, "bpd_pda_mask_bits: bad batch");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(out_bits != nullptr, "bpd_pda_mask_bits: null output");
  BPD_REQUIRE(batch <= 65535, "bpd_pda_mask_bits: batch > 65535");
  cudaStream_t st = as_stream(stream);
  Memo m;
  Work w;
  bpd_status rc = run_mask_pipeline(g, config_pool, slots, broken, batch, memo, memo_capacity,
                                    workspace, &m, &w, st);
  if (rc) return rc;
  const int32_t W = (g->vocab_size + 31) / 32;
  dim3 grid((W + 255) / 256, batch);
  pda_bits_out_kernel<<<grid, 256, 0, st>>>(W, m, w, out_bits);
  return check_launch("pda_bits_out_kernel");
}

extern "C" bpd_status bpd_pda_apply_mask(const bpd_pda_grammar* g, void* logits, int32_t dtype,
                                         int64_t row_stride, const int32_t* config_pool,
                                         const int64_t* slots, const uint8_t* broken,
                                         int32_t batch, void* memo, int32_t memo_capacity,
                                         void* workspace, float neg_inf, void* stream) {
  BPD_REQUIRE(batch >= 0, "bpd_pda_apply_mask: bad batch");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(logits != nullptr, "bpd_pda_apply_mask: null logits");
  BPD_REQUIRE(g && row_stride >= g->vocab_size, "bpd_pda_apply_mask: row_stride < vocab");
  cudaStream_t st = as_stream(stream);
  Memo m;
  Work w;
  bpd_status rc = run_mask_pipeline(g, config_pool, slots, broken, batch, memo, memo_capacity,
                                    workspace, &m, &w, st);
  if (rc) return rc;
  return with_dtype(dtype, "bpd_pda_apply_mask", [&](auto tag) {
    using T = decltype(tag);
    return launch_pda_apply<T>(logits, row_stride, batch, g->vocab_size, m, w, neg_inf, st);
  });
}

extern "C" bpd_status bpd_pda_step_greedy(
    const bpd_pda_grammar* g, void* logits, int32_t dtype, int64_t row_stride,
    int32_t* config_pool, const int64_t* slots, uint8_t* broken, int32_t batch, void* memo,
    int32_t memo_capacity, void* workspace, float neg_inf, int64_t* token_out,
    int32_t* status_out, int32_t chunks_per_row, void* stream) {
  BPD_REQUIRE(batch >= 0, "bpd_pda_step_greedy: bad batch");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(logits != nullptr && token_out != nullptr, "bpd_pda_step_greedy: null pointer");
  BPD_REQUIRE(g && row_stride >= g->vocab_size, "bpd_pda_step_greedy: row_stride < vocab");
  BPD_REQUIRE(chunks_per_row >= 0 && chunks_per_row <= 4096,
              "bpd_pda_step_greedy: chunks_per_row must be in [0, 4096]");
  cudaStream_t st = as_stream(stream);
  Memo m;
  Work w;
  bpd_status rc = run_mask_pipeline(g, config_pool, slots, broken, batch, memo, memo_capacity,
                                    workspace, &m, &w, st);
  if (rc) return rc;
  const int32_t k = chunks_per_row;
  const PdaCommit commit{*g, config_pool, slots, token_out, broken, status_out};
  return with_dtype(dtype, "bpd_pda_step_greedy", [&](auto tag) {
    using T = decltype(tag);
    return launch_pda_step<T>(logits, row_stride, batch, g->vocab_size, m, w, neg_inf, commit,
                              k, st);
  });
}

namespace bpd {
namespace {
bpd_status pda_step_from(
    const bpd_pda_grammar* g, const void* src, int32_t src_dtype, int64_t src_stride,
    const int64_t* src_rows, float* out, int64_t out_stride, int32_t* config_pool,
    const int64_t* slots, uint8_t* broken, int32_t batch, void* memo, int32_t memo_capacity,
    void* workspace, float neg_inf, int64_t* token_out, int32_t* status_out,
    int32_t chunks_per_row, void* stream, const int32_t* nrows, const char* what) {
  BPD_REQUIRE(batch >= 0, "%s: bad batch", what);
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(src != nullptr && token_out != nullptr, "%s: null pointer", what);
  BPD_REQUIRE(g && src_stride >= g->vocab_size &&
                  (out == nullptr || out_stride >= g->vocab_size),
              "%s: row stride < vocab", what);
  BPD_REQUIRE(chunks_per_row >= 0 && chunks_per_row <= 4096,
              "%s: chunks_per_row must be in [0, 4096]", what);
  cudaStream_t st = as_stream(stream);
  Memo m;
  Work w;
  bpd_status rc = run_mask_pipeline(g, config_pool, slots, broken, batch, memo, memo_capacity,
                                    workspace, &m, &w, st, nrows);
  if (rc) return rc;
  const PdaCommit commit{*g, config_pool, slots, token_out, broken, status_out};
  const PdaRows rows{m, w};
  const int32_t V = g->vocab_size;
  return with_dtype(src_dtype, what, [&](auto tag) {
    using T = decltype(tag);
    return launch_stream_step_src<T, PdaRows, PdaCommit>(
        src, src_stride, src_rows, out, out_stride, batch, V, rows, commit, neg_inf,
        chunks_per_row, w.step, st, what, nrows);
  }, "source");
}
}  // namespace
}  // namespace bpd

extern "C" bpd_status bpd_pda_step_greedy_from(
    const bpd_pda_grammar* g, const void* src, int32_t src_dtype, int64_t src_stride,
    const int64_t* src_rows, float* out, int64_t out_stride, int32_t* config_pool,
    const int64_t* slots, uint8_t* broken, int32_t batch, void* memo, int32_t memo_capacity,
    void* workspace, float neg_inf, int64_t* token_out, int32_t* status_out,
    int32_t chunks_per_row, void* stream) {
  return pda_step_from(g, src, src_dtype, src_stride, src_rows, out, out_stride, config_pool,
                       slots, broken, batch, memo, memo_capacity, workspace, neg_inf, token_out,
                       status_out, chunks_per_row, stream, nullptr, "bpd_pda_step_greedy_from");
}

extern "C" bpd_status bpd_pda_step_greedy_from_n(
    const bpd_pda_grammar* g, const void* src, int32_t src_dtype, int64_t src_stride,
    const int64_t* src_rows, float* out, int64_t out_stride, int32_t* config_pool,
    const int64_t* slots, uint8_t* broken, int32_t batch, const int32_t* batch_dev, void* memo,
    int32_t memo_capacity, void* workspace, float neg_inf, int64_t* token_out,
    int32_t* status_out, int32_t chunks_per_row, void* stream) {
  BPD_REQUIRE(batch_dev != nullptr, "bpd_pda_step_greedy_from_n: null row count");
  return pda_step_from(g, src, src_dtype, src_stride, src_rows, out, out_stride, config_pool,
                       slots, broken, batch, memo, memo_capacity, workspace, neg_inf, token_out,
                       status_out, chunks_per_row, stream, batch_dev,
                       "bpd_pda_step_greedy_from_n");
}

extern "C" bpd_status bpd_pda_advance(const bpd_pda_grammar* g, int32_t* config_pool,
                                      const int64_t* slots, int32_t batch, const void* tokens,
                                      int32_t tokens_int64, uint8_t* ok_out, uint8_t* broken,
                                      int32_t* status_out, void* stream) {
  bpd_status rc = check_grammar(g);
  if (rc) return rc;
  BPD_REQUIRE(batch >= 0, "bpd_pda_advance: bad batch");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(config_pool && tokens, "bpd_pda_advance: null pointer");
  const int32_t blocks = (batch + kAdvWarps - 1) / kAdvWarps;
  advance_kernel<<<blocks, kAdvWarps * 32, 0, as_stream(stream)>>>(
      *g, config_pool, slots, batch, tokens, tokens_int64, ok_out, broken, status_out);
  return check_launch("pda advance_kernel");
}

extern "C" bpd_status bpd_pda_is_complete(const bpd_pda_grammar* g, const int32_t* config_pool,
                                          const int64_t* slots, const uint8_t* broken,
                                          int32_t batch, uint8_t* complete_out, void* stream) {
  bpd_status rc = check_grammar(g);
  if (rc) return rc;
  BPD_REQUIRE(batch >= 0, "bpd_pda_is_complete: bad batch");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(config_pool && complete_out, "bpd_pda_is_complete: null pointer");
  complete_kernel<<<(batch + 127) / 128, 128, 0, as_stream(stream)>>>(*g, config_pool, slots,
                                                                      broken, batch, complete_out);
  return check_launch("pda complete_kernel");
}

// ---------------------------------------------------------------------------
// Allocation-free variant of bpd_pda_apply_mask (no counterpart in the
// reference). Its per-call scratch lives in one fixed device array of this
// library, sized for BPD_NOALLOC_MAX_BATCH rows of up to BPD_NOALLOC_MAX_VOCAB
// tokens; every device that loads the library holds that array until exit.

namespace bpd {
namespace {

constexpr size_t kNoAllocBytes = work_bytes(BPD_NOALLOC_MAX_BATCH, BPD_NOALLOC_MAX_VOCAB);
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
CUcontext g_noalloc_ctx[kMaxDevices] = {};  // the context each address belongs to

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;

// The calling thread's current driver context (nullptr if it has none yet),
// through the driver entry point the runtime hands out, so the library does
// not link libcuda itself.
bpd_status current_context(CUcontext* ctx) {
  if (g_ctx_get_current == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return fail(BPD_ERR_CUDA, "cudaGetDriverEntryPoint(cuCtxGetCurrent): %s",
                  cudaGetErrorString(e));
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  *ctx = nullptr;
  if (g_ctx_get_current(ctx) != CUDA_SUCCESS)
    return fail(BPD_ERR_CUDA, "cuCtxGetCurrent failed");
  return BPD_OK;
}

// Device address of g_noalloc_scratch on the current device. In host code the
// symbol itself is only a host-side stand-in, so the address is looked up
// with cudaGetSymbolAddress (with that device current) on the first call on a
// device and cached with the context it belongs to. A later call from another
// context on that device (after cudaDeviceReset, say, which unloads the
// library's module with the old context) looks the address up again.
bpd_status noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(BPD_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(BPD_ERR_CAPACITY, "bpd_pda_apply_mask_noalloc: device %d beyond %d", dev,
                kMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  CUcontext ctx = nullptr;
  bpd_status rc = current_context(&ctx);
  if (rc) return rc;
  if (g_noalloc_ptr[dev] == nullptr || ctx == nullptr || ctx != g_noalloc_ctx[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(BPD_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    rc = current_context(&ctx);  // the lookup made the device's context current
    if (rc) return rc;
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = ctx;
  }
  *out = g_noalloc_ptr[dev];
  return BPD_OK;
}

}  // namespace
}  // namespace bpd

extern "C" bpd_status bpd_pda_apply_mask_noalloc(const bpd_pda_grammar* g, void* logits,
                                                 int32_t dtype, int64_t row_stride,
                                                 const int32_t* config_pool, const int64_t* slots,
                                                 const uint8_t* broken, int32_t batch, void* memo,
                                                 int32_t memo_capacity, float neg_inf,
                                                 void* stream) {
  BPD_REQUIRE(batch >= 0, "bpd_pda_apply_mask_noalloc: bad batch");
  if (batch == 0) return BPD_OK;
  BPD_REQUIRE(g != nullptr, "bpd_pda_apply_mask_noalloc: null grammar");
  if (batch > BPD_NOALLOC_MAX_BATCH || g->vocab_size > BPD_NOALLOC_MAX_VOCAB)
    return fail(BPD_ERR_CAPACITY,
                "bpd_pda_apply_mask_noalloc: batch %d / vocab %d exceed the built-in scratch "
                "(at most %d rows of %d tokens); use bpd_pda_apply_mask with a workspace",
                batch, g->vocab_size, BPD_NOALLOC_MAX_BATCH, BPD_NOALLOC_MAX_VOCAB);
  void* scratch = nullptr;
  const bpd_status rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  return bpd_pda_apply_mask(g, logits, dtype, row_stride, config_pool, slots, broken, batch,
                            memo, memo_capacity, scratch, neg_inf, stream);
}
