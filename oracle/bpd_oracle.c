/*
 * bpd_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, single-threaded restatement of bpdecode's constrained-decoding
 * step, used as the parity checker for the CUDA path (and, timed, as the CPU
 * baseline). Nothing in the product links or calls this file: only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg load it.
 *
 * Each function cites the reference source it restates. The PDA functions keep
 * the reference's literal control flow (round-based closure, push order,
 * saturation, prune compaction, whole-struct copies) so that full 266-int
 * config rows -- including words outside the live region -- compare equal.
 *
 * Parity of this file is pinned against (a) the reference's own C++ sources
 * compiled unchanged into oracle/_ref/ (see oracle/Makefile), and (b) golden
 * vectors generated from the reference's Python package (tests/golden/).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* Dense regular path                                                        */
/* ------------------------------------------------------------------------ */

/* mask_cpu.cpp:51-67 (step). */
int32_t orc_step(const int32_t* trans, int32_t num_symbols, const uint8_t* accept,
                 const uint8_t* live, int32_t dead, const int32_t* offsets,
                 const int32_t* symbols, int32_t eos_id, int32_t state, int32_t tok) {
  if (tok == eos_id) return (state >= 0 && accept[state]) ? state : -1;
  if (state < 0) return -1;
  int32_t cur = state;
  for (int32_t i = offsets[tok]; i < offsets[tok + 1]; ++i) {
    const int32_t sym = symbols[i];
    if (sym < 0 || sym >= num_symbols) return -1;
    cur = trans[(int64_t)cur * num_symbols + sym];
    if (cur == dead) return -1;
  }
  return live[cur] ? cur : -1;
}

/* ops.py:143-197 (build_token_transitions): tok_next[s, t] == step(s, t), the
 * equivalence the reference pins in tests/test_dense.py:42-52. */
void orc_build_tok_next(const int32_t* trans, int32_t num_states, int32_t num_symbols,
                        const uint8_t* accept, const uint8_t* live, int32_t dead,
                        const int32_t* offsets, const int32_t* symbols, int32_t vocab,
                        int32_t eos_id, int32_t* out) {
  for (int32_t s = 0; s < num_states; ++s)
    for (int32_t t = 0; t < vocab; ++t)
      out[(int64_t)s * vocab + t] =
          orc_step(trans, num_symbols, accept, live, dead, offsets, symbols, eos_id, s, t);
}

/* Packed allow bits, LSB first (mask_cpu.cpp:69-81 bit layout). */
void orc_allow_bits(const int32_t* tok_next, int32_t num_states, int32_t vocab,
                    int32_t words_stride, uint32_t* out) {
  memset(out, 0, sizeof(uint32_t) * (size_t)num_states * (size_t)words_stride);
  for (int32_t s = 0; s < num_states; ++s)
    for (int32_t t = 0; t < vocab; ++t)
      if (tok_next[(int64_t)s * vocab + t] != -1)
        out[(int64_t)s * words_stride + (t >> 5)] |= 1u << (t & 31);
}

static int state_ok(int32_t s, int32_t num_states) { return s >= 0 && s < num_states; }

/* ops.py:271-276: rejected = tok_next[max(s,0)] == -1, rejected |= s < 0. */
void orc_dense_apply_mask_f32(float* logits, int64_t row_stride, int32_t batch,
                              int32_t vocab, const int32_t* tok_next, int32_t num_states,
                              const int32_t* states, float neg_inf) {
  for (int32_t b = 0; b < batch; ++b) {
    float* row = logits + (int64_t)b * row_stride;
    const int32_t s = states[b];
    for (int32_t t = 0; t < vocab; ++t)
      if (!state_ok(s, num_states) || tok_next[(int64_t)s * vocab + t] == -1) row[t] = neg_inf;
  }
}

/* Same, for 16-bit logits (bf16 / fp16): the fill value is the caller's
 * neg_inf already rounded to the logits dtype. */
void orc_dense_apply_mask_u16(uint16_t* logits, int64_t row_stride, int32_t batch,
                              int32_t vocab, const int32_t* tok_next, int32_t num_states,
                              const int32_t* states, uint16_t neg_inf_bits) {
  for (int32_t b = 0; b < batch; ++b) {
    uint16_t* row = logits + (int64_t)b * row_stride;
    const int32_t s = states[b];
    for (int32_t t = 0; t < vocab; ++t)
      if (!state_ok(s, num_states) || tok_next[(int64_t)s * vocab + t] == -1)
        row[t] = neg_inf_bits;
  }
}

/* ops.py:301-306: next = s < 0 ? -1 : tok_next[s, t]. */
void orc_dense_advance(const int32_t* tok_next, int32_t num_states, int32_t vocab,
                       const int32_t* states, const int64_t* tokens, int32_t batch,
                       int32_t* out) {
  for (int32_t b = 0; b < batch; ++b) {
    const int32_t s = states[b];
    const int64_t t = tokens[b];
    out[b] = (!state_ok(s, num_states) || t < 0 || t >= vocab) ? -1
                                                               : tok_next[(int64_t)s * vocab + t];
  }
}

/* compute_mask (mask_cpu.cpp:69-90) over the dense table. */
void orc_dense_mask_bits(const int32_t* tok_next, int32_t num_states, int32_t vocab,
                         const int32_t* states, int32_t batch, uint32_t* out) {
  const int32_t words = (vocab + 31) / 32;
  memset(out, 0, sizeof(uint32_t) * (size_t)batch * (size_t)words);
  for (int32_t b = 0; b < batch; ++b) {
    const int32_t s = states[b];
    if (!state_ok(s, num_states)) continue;
    for (int32_t t = 0; t < vocab; ++t)
      if (tok_next[(int64_t)s * vocab + t] != -1)
        out[(int64_t)b * words + (t >> 5)] |= 1u << (t & 31);
  }
}

/* ------------------------------------------------------------------------ */
/* Soft lookahead                                                            */
/* ------------------------------------------------------------------------ */

static double lse_pair(double a, double b) {
  if (isinf(a) && a < 0) return b;
  if (isinf(b) && b < 0) return a;
  const double m = a > b ? a : b;
  return m + log(exp(a - m) + exp(b - m));
}

/* ops.py:200-236, in double precision: logZ_0 = live ? 0 : -inf; k-1 rounds of
 * logZ(s) = live ? LSE_t logZ[tn[s,t]] (LSE with 0 if accepting) : -inf, with
 * the EOS column of tok_next (= s when accepting) inside the sum like the
 * reference; out[s,t] = logZ[tn[s,t]] or -inf; EOS column 0 / -inf. */
void orc_build_lookahead(const int32_t* tok_next, int32_t num_states, int32_t vocab,
                         const uint8_t* accept, const uint8_t* live, int32_t eos_id,
                         int32_t k, double* logz_work, double* logz_next, double* out) {
  for (int32_t s = 0; s < num_states; ++s) logz_work[s] = live[s] ? 0.0 : -INFINITY;
  for (int32_t r = 0; r < (k - 1 > 0 ? k - 1 : 0); ++r) {
    for (int32_t s = 0; s < num_states; ++s) {
      double m = -INFINITY;
      for (int32_t t = 0; t < vocab; ++t) {
        const int32_t n = tok_next[(int64_t)s * vocab + t];
        if (n >= 0 && logz_work[n] > m) m = logz_work[n];
      }
      double acc = -INFINITY;
      if (!(isinf(m) && m < 0)) {
        double sum = 0.0;
        for (int32_t t = 0; t < vocab; ++t) {
          const int32_t n = tok_next[(int64_t)s * vocab + t];
          if (n >= 0) sum += exp(logz_work[n] - m);
        }
        acc = m + log(sum);
      }
      if (accept[s]) acc = lse_pair(acc, 0.0);
      logz_next[s] = live[s] ? acc : -INFINITY;
    }
    memcpy(logz_work, logz_next, sizeof(double) * (size_t)num_states);
  }
  for (int32_t s = 0; s < num_states; ++s) {
    for (int32_t t = 0; t < vocab; ++t) {
      const int32_t n = tok_next[(int64_t)s * vocab + t];
      out[(int64_t)s * vocab + t] = n >= 0 ? logz_work[n] : -INFINITY;
    }
    if (eos_id >= 0 && eos_id < vocab)
      out[(int64_t)s * vocab + eos_id] = accept[s] ? 0.0 : -INFINITY;
  }
}

/* ops.py:239-259 (apply_soft_), fp32 logits. */
void orc_apply_soft_f32(float* logits, int64_t row_stride, int32_t batch, int32_t vocab,
                        const float* lookahead, int32_t num_states, const int32_t* states,
                        float alpha) {
  for (int32_t b = 0; b < batch; ++b) {
    float* row = logits + (int64_t)b * row_stride;
    const int32_t s = states[b];
    for (int32_t t = 0; t < vocab; ++t) {
      const float bias = state_ok(s, num_states) ? lookahead[(int64_t)s * vocab + t] : -INFINITY;
      const int disallowed = isinf(bias) && bias < 0;
      if (alpha != 0.0f) row[t] = row[t] + alpha * (disallowed ? 0.0f : bias);
      if (disallowed) row[t] = -INFINITY;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Pushdown automaton                                                        */
/* ------------------------------------------------------------------------ */

#define MC 8
#define MD 32
#define NCFG (2 + MC + MC * MD)
#define NUM(c) ((c)[0])
#define SAT(c) ((c)[1])
#define DEPTH(c, i) ((c)[2 + (i)])
#define STACK(c, i) ((c) + 2 + MC + (i) * MD)

enum { EDGE_EPS = 0, EDGE_BYTE = 1, EDGE_CALL = 2 };

typedef struct orc_pda_grammar {
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
} orc_pda_grammar;

/* pda.hpp:95-108 */
static int stack_eq(const int32_t* a, const int32_t* b, int32_t n) {
  for (int32_t i = 0; i < n; ++i)
    if (a[i] != b[i]) return 0;
  return 1;
}
static int contains(const int32_t* c, const int32_t* st, int32_t depth) {
  for (int32_t i = 0; i < NUM(c); ++i)
    if (DEPTH(c, i) == depth && stack_eq(STACK(c, i), st, depth)) return 1;
  return 0;
}

/* pda.hpp:111-121 */
static int push(int32_t* c, const int32_t* st, int32_t depth) {
  if (NUM(c) >= MC) {
    SAT(c) = 1;
    return 0;
  }
  const int32_t i = NUM(c)++;
  DEPTH(c, i) = depth;
  for (int32_t k = 0; k < depth; ++k) STACK(c, i)[k] = st[k];
  return 1;
}

/* pda.hpp:124-139 */
static void prune_dead(const orc_pda_grammar* g, int32_t* c) {
  int32_t out = 0;
  for (int32_t i = 0; i < NUM(c); ++i) {
    const int32_t d = DEPTH(c, i);
    if (d <= 0) continue;
    if (!g->live[STACK(c, i)[d - 1]]) continue;
    if (out != i) {
      DEPTH(c, out) = d;
      for (int32_t k = 0; k < d; ++k) STACK(c, out)[k] = STACK(c, i)[k];
    }
    ++out;
  }
  NUM(c) = out;
}

/* pda.hpp:150-198: rounds until no push succeeds (guard 8*32+8). */
static int close_set(const orc_pda_grammar* g, int32_t* c) {
  int changed = 1;
  int32_t guard = 0;
  const int32_t max_rounds = MC * MD + 8;
  while (changed && guard++ < max_rounds) {
    changed = 0;
    const int32_t n = NUM(c);
    for (int32_t i = 0; i < n; ++i) {
      const int32_t d = DEPTH(c, i);
      if (d <= 0) continue;
      const int32_t top = STACK(c, i)[d - 1];
      if (g->accept[top] && d > 1) {
        if (!contains(c, STACK(c, i), d - 1) && push(c, STACK(c, i), d - 1)) changed = 1;
      }
      for (int32_t e = g->edge_offsets[top]; e < g->edge_offsets[top + 1]; ++e) {
        const int32_t kind = g->edge_kind[e];
        if (kind == EDGE_EPS) {
          int32_t tmp[MD];
          for (int32_t k = 0; k < d - 1; ++k) tmp[k] = STACK(c, i)[k];
          tmp[d - 1] = g->edge_dst[e];
          if (!contains(c, tmp, d) && push(c, tmp, d)) changed = 1;
        } else if (kind == EDGE_CALL) {
          if (d + 1 <= MD) {
            int32_t tmp[MD];
            for (int32_t k = 0; k < d - 1; ++k) tmp[k] = STACK(c, i)[k];
            tmp[d - 1] = g->edge_dst[e];
            tmp[d] = g->edge_callee[e];
            if (!contains(c, tmp, d + 1) && push(c, tmp, d + 1)) changed = 1;
          } else {
            SAT(c) = 1;
          }
        }
      }
    }
  }
  prune_dead(g, c);
  return NUM(c) > 0;
}

/* pda.hpp:200-207 (on a zero-initialised struct, as pda_init_op does). */
void orc_pda_init(const orc_pda_grammar* g, int32_t* cfg_out) {
  memset(cfg_out, 0, sizeof(int32_t) * NCFG);
  int32_t st[1] = {g->root_start};
  push(cfg_out, st, 1);
  close_set(g, cfg_out);
}

/* pda.hpp:211-236 */
static int advance_byte(const orc_pda_grammar* g, int32_t* c, int32_t byte) {
  int32_t next[NCFG];
  memset(next, 0, sizeof(next));
  for (int32_t i = 0; i < NUM(c); ++i) {
    const int32_t d = DEPTH(c, i);
    if (d <= 0) continue;
    const int32_t top = STACK(c, i)[d - 1];
    for (int32_t e = g->edge_offsets[top]; e < g->edge_offsets[top + 1]; ++e) {
      if (g->edge_kind[e] != EDGE_BYTE) continue;
      if (byte < g->edge_lo[e] || byte > g->edge_hi[e]) continue;
      int32_t tmp[MD];
      for (int32_t k = 0; k < d - 1; ++k) tmp[k] = STACK(c, i)[k];
      tmp[d - 1] = g->edge_dst[e];
      if (!contains(next, tmp, d)) push(next, tmp, d);
    }
  }
  SAT(next) = SAT(next) || SAT(c);
  const int ok = close_set(g, next);
  memcpy(c, next, sizeof(next));
  return ok;
}

/* pda.hpp:238-244 */
int orc_pda_is_complete(const orc_pda_grammar* g, const int32_t* c) {
  for (int32_t i = 0; i < NUM(c); ++i)
    if (DEPTH(c, i) == 1 && STACK(c, i)[0] == g->root_accept) return 1;
  return 0;
}

/* pda.hpp:248-258 */
int orc_pda_try_token(const orc_pda_grammar* g, const int32_t* cfg, int32_t tok) {
  if (tok == g->eos_id) return orc_pda_is_complete(g, cfg);
  int32_t c[NCFG];
  memcpy(c, cfg, sizeof(c));
  for (int32_t i = g->tok_offsets[tok]; i < g->tok_offsets[tok + 1]; ++i)
    if (!advance_byte(g, c, g->tok_bytes[i])) return 0;
  return NUM(c) > 0;
}

/* Advance one config-set by one byte in place (the reference's feed() helper,
 * csrc/tests/test_pda.cpp:47-52, one byte at a time). */
int orc_pda_advance_byte(const orc_pda_grammar* g, int32_t* cfg, int32_t byte) {
  return advance_byte(g, cfg, byte);
}

/* pda_cpu.cpp:7-21 */
void orc_pda_mask_bits(const orc_pda_grammar* g, const int32_t* cfgs, int32_t batch,
                       uint32_t* out) {
  const int32_t words = (g->vocab_size + 31) / 32;
  memset(out, 0, sizeof(uint32_t) * (size_t)batch * (size_t)words);
  for (int32_t b = 0; b < batch; ++b) {
    const int32_t* c = cfgs + (int64_t)b * NCFG;
    uint32_t* row = out + (int64_t)b * words;
    for (int32_t t = 0; t < g->vocab_size; ++t)
      if (orc_pda_try_token(g, c, t)) row[t >> 5] |= 1u << (t & 31);
    if (g->eos_id >= 0 && orc_pda_is_complete(g, c))
      row[g->eos_id >> 5] |= 1u << (g->eos_id & 31);
  }
}

/* pda_cpu.cpp:23-33 */
void orc_pda_apply_mask_f32(const orc_pda_grammar* g, const int32_t* cfgs, int32_t batch,
                            float* logits, int64_t row_stride, float neg_inf) {
  for (int32_t b = 0; b < batch; ++b) {
    float* row = logits + (int64_t)b * row_stride;
    for (int32_t t = 0; t < g->vocab_size; ++t)
      if (!orc_pda_try_token(g, cfgs + (int64_t)b * NCFG, t)) row[t] = neg_inf;
  }
}

/* pda_cpu.cpp:35-54 */
void orc_pda_advance(const orc_pda_grammar* g, int32_t* cfgs, const int64_t* tokens,
                     int32_t batch, uint8_t* ok) {
  for (int32_t b = 0; b < batch; ++b) {
    int32_t* c = cfgs + (int64_t)b * NCFG;
    const int32_t t = (int32_t)tokens[b];
    if (t == g->eos_id) {
      ok[b] = (uint8_t)orc_pda_is_complete(g, c);
      continue;
    }
    int32_t trial[NCFG];
    memcpy(trial, c, sizeof(trial));
    int accepted = 1;
    for (int32_t i = g->tok_offsets[t]; i < g->tok_offsets[t + 1] && accepted; ++i)
      accepted = advance_byte(g, trial, g->tok_bytes[i]);
    ok[b] = (uint8_t)accepted;
    if (accepted) memcpy(c, trial, sizeof(trial));
  }
}
