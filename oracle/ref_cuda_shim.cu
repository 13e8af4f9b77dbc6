// ref_cuda_shim.cu -- TEST INFRASTRUCTURE ONLY.
//
// extern "C" wrappers over the reference's own CUDA implementation
// (csrc/src/mask_cuda.cu and csrc/src/pda_cuda.cu, which run the header-only
// primitives of csrc/include/bpdecode/{mask,pda}.hpp on the device), compiled
// unchanged from the reference tree for sm_100a by oracle/Makefile into
// oracle/_ref/libbpdref_cuda.so. Every pointer is a device pointer, every
// launch goes to `stream` and nothing synchronises -- the reference's own
// contract (bindings/torch_ops.cpp hands it raw tensor pointers the same way).
// The declarations restate the launchers' signatures (mask_cuda.cu:175-236,
// pda_cuda.cu:127-188); the library defines them.
#include <cstdint>

#include "bpdecode/pda.hpp"

namespace bpdecode {

void compute_mask_batch_cuda(int32_t num_states, int32_t num_symbols, const int32_t* trans,
                             const uint8_t* accept, const uint8_t* live, int32_t dead,
                             const int32_t* offsets, const int32_t* symbols, int32_t vocab_size,
                             int32_t eos_id, const int32_t* states, int32_t batch,
                             uint32_t* out_bits, void* stream);

void advance_state_batch_cuda(int32_t num_states, int32_t num_symbols, const int32_t* trans,
                              const uint8_t* accept, const uint8_t* live, int32_t dead,
                              const int32_t* offsets, const int32_t* symbols,
                              int32_t vocab_size, int32_t eos_id, const int32_t* states,
                              const int32_t* token_ids, int32_t batch, int32_t* next_states,
                              void* stream);

void compute_mask_pda_batch_cuda(int32_t num_states, int32_t root_start, int32_t root_accept,
                                 const uint8_t* accept, const uint8_t* live,
                                 const int32_t* edge_offsets, const int32_t* edge_kind,
                                 const int32_t* edge_lo, const int32_t* edge_hi,
                                 const int32_t* edge_dst, const int32_t* edge_callee,
                                 int32_t vocab_size, int32_t eos_id, const int32_t* tok_offsets,
                                 const uint8_t* tok_bytes, const PdaConfigSet* configs,
                                 int32_t batch, uint32_t* out_bits, void* stream);

void apply_mask_pda_batch_cuda(int32_t num_states, int32_t root_start, int32_t root_accept,
                               const uint8_t* accept, const uint8_t* live,
                               const int32_t* edge_offsets, const int32_t* edge_kind,
                               const int32_t* edge_lo, const int32_t* edge_hi,
                               const int32_t* edge_dst, const int32_t* edge_callee,
                               int32_t vocab_size, int32_t eos_id, const int32_t* tok_offsets,
                               const uint8_t* tok_bytes, const PdaConfigSet* configs,
                               int32_t batch, float* logits, float neg_inf, void* stream);

void advance_state_pda_batch_cuda(int32_t num_states, int32_t root_start, int32_t root_accept,
                                  const uint8_t* accept, const uint8_t* live,
                                  const int32_t* edge_offsets, const int32_t* edge_kind,
                                  const int32_t* edge_lo, const int32_t* edge_hi,
                                  const int32_t* edge_dst, const int32_t* edge_callee,
                                  int32_t vocab_size, int32_t eos_id,
                                  const int32_t* tok_offsets, const uint8_t* tok_bytes,
                                  PdaConfigSet* configs, const int32_t* token_ids, int32_t batch,
                                  uint8_t* ok, void* stream);

}  // namespace bpdecode

using namespace bpdecode;

// The PDA grammar tables as the reference's launchers take them.
struct RefPda {
  int32_t num_states, root_start, root_accept;
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

extern "C" {

int32_t bpdref_cuda_config_bytes() { return static_cast<int32_t>(sizeof(PdaConfigSet)); }

void bpdref_cuda_compute_mask(int32_t num_states, int32_t num_symbols, const int32_t* trans,
                              const uint8_t* accept, const uint8_t* live, int32_t dead,
                              const int32_t* offsets, const int32_t* symbols, int32_t vocab,
                              int32_t eos_id, const int32_t* states, int32_t batch,
                              uint32_t* out_bits, void* stream) {
  compute_mask_batch_cuda(num_states, num_symbols, trans, accept, live, dead, offsets, symbols,
                          vocab, eos_id, states, batch, out_bits, stream);
}

void bpdref_cuda_advance_state(int32_t num_states, int32_t num_symbols, const int32_t* trans,
                               const uint8_t* accept, const uint8_t* live, int32_t dead,
                               const int32_t* offsets, const int32_t* symbols, int32_t vocab,
                               int32_t eos_id, const int32_t* states, const int32_t* tokens,
                               int32_t batch, int32_t* next_states, void* stream) {
  advance_state_batch_cuda(num_states, num_symbols, trans, accept, live, dead, offsets, symbols,
                           vocab, eos_id, states, tokens, batch, next_states, stream);
}

void bpdref_cuda_pda_mask(const RefPda* g, const int32_t* configs, int32_t batch,
                          uint32_t* out_bits, void* stream) {
  compute_mask_pda_batch_cuda(g->num_states, g->root_start, g->root_accept, g->accept, g->live,
                              g->edge_offsets, g->edge_kind, g->edge_lo, g->edge_hi,
                              g->edge_dst, g->edge_callee, g->vocab_size, g->eos_id,
                              g->tok_offsets, g->tok_bytes,
                              reinterpret_cast<const PdaConfigSet*>(configs), batch, out_bits,
                              stream);
}

void bpdref_cuda_pda_apply_mask(const RefPda* g, const int32_t* configs, int32_t batch,
                                float* logits, float neg_inf, void* stream) {
  apply_mask_pda_batch_cuda(g->num_states, g->root_start, g->root_accept, g->accept, g->live,
                            g->edge_offsets, g->edge_kind, g->edge_lo, g->edge_hi, g->edge_dst,
                            g->edge_callee, g->vocab_size, g->eos_id, g->tok_offsets,
                            g->tok_bytes, reinterpret_cast<const PdaConfigSet*>(configs), batch,
                            logits, neg_inf, stream);
}

void bpdref_cuda_pda_advance(const RefPda* g, int32_t* configs, const int32_t* tokens,
                             int32_t batch, uint8_t* ok, void* stream) {
  advance_state_pda_batch_cuda(g->num_states, g->root_start, g->root_accept, g->accept, g->live,
                               g->edge_offsets, g->edge_kind, g->edge_lo, g->edge_hi,
                               g->edge_dst, g->edge_callee, g->vocab_size, g->eos_id,
                               g->tok_offsets, g->tok_bytes,
                               reinterpret_cast<PdaConfigSet*>(configs), tokens, batch, ok,
                               stream);
}

}  // extern "C"
