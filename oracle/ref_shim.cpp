// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// extern "C" wrappers over the reference's own CPU implementation
// (csrc/src/mask_cpu.cpp, csrc/src/pda_cpu.cpp and the header-only PDA
// primitives of csrc/include/bpdecode/pda.hpp), compiled unchanged from the
// reference tree by oracle/Makefile into oracle/_ref/libbpdref.so. The
// wrappers only marshal plain arrays into the reference's FsaTable / PdaTable
// structs, the way its torch binding does (bindings/torch_ops.cpp:54-86,
// 249-298), so Python tests can drive the reference through ctypes.
#include <cstdint>
#include <cstring>

#include "bpdecode/mask.hpp"
#include "bpdecode/pda.hpp"

using namespace bpdecode;

namespace {

FsaTable make_fsa(const int32_t* trans, int32_t num_states, int32_t num_symbols,
                  const uint8_t* accept, const uint8_t* live, int32_t dead) {
  FsaTable f;
  f.num_states = num_states;
  f.num_symbols = num_symbols;
  f.start = 0;
  f.dead = dead;
  f.trans.assign(trans, trans + static_cast<int64_t>(num_states) * num_symbols);
  f.accept.assign(accept, accept + num_states);
  if (live) f.live.assign(live, live + num_states);
  return f;
}

TokenSymbols make_toks(const int32_t* offsets, const int32_t* symbols, int32_t vocab,
                       int32_t eos_id) {
  TokenSymbols t;
  t.vocab_size = vocab;
  t.eos_id = eos_id;
  t.offsets.assign(offsets, offsets + vocab + 1);
  t.symbols.assign(symbols, symbols + offsets[vocab]);
  return t;
}

// Same field layout as orc_pda_grammar / bpd_pda_grammar.
struct PdaArgs {
  int32_t num_states, num_edges, root_start, root_accept;
  const uint8_t* accept;
  const uint8_t* live;
  const int32_t* edge_offsets;
  const int32_t* edge_kind;
  const int32_t* edge_lo;
  const int32_t* edge_hi;
  const int32_t* edge_dst;
  const int32_t* edge_callee;
  int32_t vocab_size, eos_id;
  const int32_t* tok_offsets;
  const uint8_t* tok_bytes;
};

PdaTable make_pda(const PdaArgs* a) {
  PdaTable g;
  g.num_states = a->num_states;
  g.root_start = a->root_start;
  g.root_accept = a->root_accept;
  g.accept.assign(a->accept, a->accept + a->num_states);
  g.live.assign(a->live, a->live + a->num_states);
  g.edge_offsets.assign(a->edge_offsets, a->edge_offsets + a->num_states + 1);
  g.edge_kind.assign(a->edge_kind, a->edge_kind + a->num_edges);
  g.edge_lo.assign(a->edge_lo, a->edge_lo + a->num_edges);
  g.edge_hi.assign(a->edge_hi, a->edge_hi + a->num_edges);
  g.edge_dst.assign(a->edge_dst, a->edge_dst + a->num_edges);
  g.edge_callee.assign(a->edge_callee, a->edge_callee + a->num_edges);
  return g;
}

PdaTokens make_pda_toks(const PdaArgs* a) {
  PdaTokens t;
  t.vocab_size = a->vocab_size;
  t.eos_id = a->eos_id;
  t.offsets.assign(a->tok_offsets, a->tok_offsets + a->vocab_size + 1);
  t.bytes.assign(a->tok_bytes, a->tok_bytes + a->tok_offsets[a->vocab_size]);
  return t;
}

}  // namespace

extern "C" {

void ref_build_reachability(const int32_t* trans, int32_t num_states, int32_t num_symbols,
                            const uint8_t* accept, uint8_t* live_out) {
  FsaTable f = make_fsa(trans, num_states, num_symbols, accept, nullptr, num_states - 1);
  build_reachability(f);
  std::memcpy(live_out, f.live.data(), static_cast<size_t>(num_states));
}

void ref_compute_mask_batch(const int32_t* trans, int32_t num_states, int32_t num_symbols,
                            const uint8_t* accept, const uint8_t* live, int32_t dead,
                            const int32_t* offsets, const int32_t* symbols, int32_t vocab,
                            int32_t eos_id, const int32_t* states, int32_t batch,
                            uint32_t* out_bits) {
  FsaTable f = make_fsa(trans, num_states, num_symbols, accept, live, dead);
  TokenSymbols t = make_toks(offsets, symbols, vocab, eos_id);
  compute_mask_batch(f, t, states, batch, out_bits);
}

void ref_advance_state_batch(const int32_t* trans, int32_t num_states, int32_t num_symbols,
                             const uint8_t* accept, const uint8_t* live, int32_t dead,
                             const int32_t* offsets, const int32_t* symbols, int32_t vocab,
                             int32_t eos_id, const int32_t* states, const int32_t* tokens,
                             int32_t batch, int32_t* next) {
  FsaTable f = make_fsa(trans, num_states, num_symbols, accept, live, dead);
  TokenSymbols t = make_toks(offsets, symbols, vocab, eos_id);
  advance_state_batch(f, t, states, tokens, batch, next);
}

void ref_apply_mask_batch(const int32_t* trans, int32_t num_states, int32_t num_symbols,
                          const uint8_t* accept, const uint8_t* live, int32_t dead,
                          const int32_t* offsets, const int32_t* symbols, int32_t vocab,
                          int32_t eos_id, const int32_t* states, int32_t batch, float* logits,
                          float neg_inf) {
  FsaTable f = make_fsa(trans, num_states, num_symbols, accept, live, dead);
  TokenSymbols t = make_toks(offsets, symbols, vocab, eos_id);
  apply_mask_batch(f, t, states, batch, logits, neg_inf);
}

void ref_pda_init(const PdaArgs* a, int32_t* cfg_out) {
  PdaTable g = make_pda(a);
  PdaConfigSet cfg;
  pda_init(g, cfg);
  std::memcpy(cfg_out, &cfg, sizeof(cfg));
}

int32_t ref_pda_is_complete(const PdaArgs* a, const int32_t* cfg) {
  PdaTable g = make_pda(a);
  PdaConfigSet c;
  std::memcpy(&c, cfg, sizeof(c));
  return pda_is_complete(g, c) ? 1 : 0;
}

int32_t ref_pda_advance_byte(const PdaArgs* a, int32_t* cfg, int32_t byte) {
  PdaTable g = make_pda(a);
  PdaConfigSet c;
  std::memcpy(&c, cfg, sizeof(c));
  const bool ok = pda_advance_byte(g, c, byte);
  std::memcpy(cfg, &c, sizeof(c));
  return ok ? 1 : 0;
}

void ref_pda_mask_bits(const PdaArgs* a, const int32_t* cfgs, int32_t batch, uint32_t* out) {
  PdaTable g = make_pda(a);
  PdaTokens t = make_pda_toks(a);
  compute_mask_pda_batch(g, t, reinterpret_cast<const PdaConfigSet*>(cfgs), batch, out);
}

void ref_pda_apply_mask(const PdaArgs* a, const int32_t* cfgs, int32_t batch, float* logits,
                        float neg_inf) {
  PdaTable g = make_pda(a);
  PdaTokens t = make_pda_toks(a);
  apply_mask_pda_batch(g, t, reinterpret_cast<const PdaConfigSet*>(cfgs), batch, logits,
                       neg_inf);
}

void ref_pda_advance(const PdaArgs* a, int32_t* cfgs, const int32_t* tokens, int32_t batch,
                     uint8_t* ok) {
  PdaTable g = make_pda(a);
  PdaTokens t = make_pda_toks(a);
  advance_state_pda_batch(g, t, reinterpret_cast<PdaConfigSet*>(cfgs), tokens, batch, ok);
}

}  // extern "C"
