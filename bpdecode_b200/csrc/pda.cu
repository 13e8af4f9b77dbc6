// Pushdown-automaton kernels (placeholder: entry points not yet implemented).
#include "common.cuh"

using namespace bpd;

extern "C" bpd_status bpd_pda_init(const bpd_pda_grammar*, int32_t*, void*) {
  return fail(BPD_ERR_INVALID, "bpd_pda_init: not implemented");
}
extern "C" size_t bpd_pda_memo_bytes(int32_t, int32_t) { return 0; }
extern "C" bpd_status bpd_pda_memo_reset(void*, int32_t, int32_t, void*) {
  return fail(BPD_ERR_INVALID, "bpd_pda_memo_reset: not implemented");
}
extern "C" size_t bpd_pda_workspace_bytes(int32_t, int32_t) { return 0; }
extern "C" bpd_status bpd_pda_mask_bits(const bpd_pda_grammar*, const int32_t*, const int64_t*,
                                        const uint8_t*, int32_t, void*, int32_t, void*, uint32_t*,
                                        void*) {
  return fail(BPD_ERR_INVALID, "bpd_pda_mask_bits: not implemented");
}
extern "C" bpd_status bpd_pda_apply_mask(const bpd_pda_grammar*, void*, int32_t, int64_t,
                                         const int32_t*, const int64_t*, const uint8_t*, int32_t,
                                         void*, int32_t, void*, float, void*) {
  return fail(BPD_ERR_INVALID, "bpd_pda_apply_mask: not implemented");
}
extern "C" bpd_status bpd_pda_advance(const bpd_pda_grammar*, int32_t*, const int64_t*, int32_t,
                                      const void*, int32_t, uint8_t*, uint8_t*, int32_t*, void*) {
  return fail(BPD_ERR_INVALID, "bpd_pda_advance: not implemented");
}
extern "C" bpd_status bpd_pda_is_complete(const bpd_pda_grammar*, const int32_t*, const int64_t*,
                                          const uint8_t*, int32_t, uint8_t*, void*) {
  return fail(BPD_ERR_INVALID, "bpd_pda_is_complete: not implemented");
}
