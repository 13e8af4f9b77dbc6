"""``torch.ops.bpdecode.*`` -- the reference's op schemas over this library.

Drop-in for ``bindings/torch_ops.cpp``: importing this module registers the
seven ops under the ``bpdecode`` namespace with the reference's exact schemas
(bindings/torch_ops.cpp:427-459), so code that calls ``torch.ops.bpdecode.*``
directly keeps working. The device ops are registered for the CUDA dispatch
key only and call the C ABI; a CPU tensor reaches no implementation and torch
raises -- there is no CPU fallback on the device path. ``build_reachability``
is the reference's host-only compile-time op and stays host-only here
(bindings/torch_ops.cpp:88-107).

The reference's own extension registers the same namespace; load one or the
other in a process, not both.
"""

from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _capi
from .ops import _check_logits, _require_cuda, _stream, _tokens

PDA_CONFIG_FLAT = 266

SCHEMAS = {
    "build_reachability": "build_reachability(Tensor trans, Tensor accept, int num_symbols) -> Tensor",
    "apply_mask_": (
        "apply_mask_(Tensor(a!) logits, Tensor trans, Tensor accept, Tensor live, "
        "int num_symbols, int dead, Tensor offsets, Tensor symbols, int eos_id, "
        "Tensor states, float neg_inf) -> Tensor(a!)"),
    "compute_mask": (
        "compute_mask(Tensor trans, Tensor accept, Tensor live, int num_symbols, "
        "int dead, Tensor offsets, Tensor symbols, int eos_id, Tensor states) -> Tensor"),
    "advance_state": (
        "advance_state(Tensor trans, Tensor accept, Tensor live, int num_symbols, "
        "int dead, Tensor offsets, Tensor symbols, int eos_id, Tensor states, "
        "Tensor token_ids) -> Tensor"),
    "pda_init": (
        "pda_init(Tensor accept, Tensor live, Tensor edge_offsets, Tensor edge_kind, "
        "Tensor edge_lo, Tensor edge_hi, Tensor edge_dst, Tensor edge_callee, "
        "int root_start, int root_accept) -> Tensor"),
    "pda_apply_mask_": (
        "pda_apply_mask_(Tensor(a!) logits, Tensor accept, Tensor live, "
        "Tensor edge_offsets, Tensor edge_kind, Tensor edge_lo, Tensor edge_hi, "
        "Tensor edge_dst, Tensor edge_callee, int root_start, int root_accept, "
        "Tensor tok_offsets, Tensor tok_bytes, int eos_id, Tensor configs, "
        "float neg_inf) -> Tensor(a!)"),
    "pda_advance_state": (
        "pda_advance_state(Tensor(a!) configs, Tensor accept, Tensor live, "
        "Tensor edge_offsets, Tensor edge_kind, Tensor edge_lo, Tensor edge_hi, "
        "Tensor edge_dst, Tensor edge_callee, int root_start, int root_accept, "
        "Tensor tok_offsets, Tensor tok_bytes, int eos_id, Tensor token_ids) -> Tensor"),
}

_LIB: torch.library.Library | None = None


def _c(t: torch.Tensor, dtype: torch.dtype, what: str) -> torch.Tensor:
    _require_cuda(t, what)
    if t.dtype != dtype:
        raise RuntimeError(f"bpdecode: {what} must be {dtype}")
    return t.contiguous()


def _dfa(trans, accept, live, num_symbols, dead, offsets, symbols, eos_id):
    tr = _c(trans, torch.int32, "trans")
    ac = _c(accept, torch.uint8, "accept")
    lv = _c(live, torch.uint8, "live")
    of = _c(offsets, torch.int32, "offsets")
    sy = _c(symbols, torch.int32, "symbols")
    if sy.numel() == 0:
        sy = torch.zeros(1, dtype=torch.int32, device=tr.device)
    keep = (tr, ac, lv, of, sy)
    args = (tr.data_ptr(), int(ac.numel()), int(num_symbols), ac.data_ptr(), lv.data_ptr(),
            int(dead), of.data_ptr(), sy.data_ptr(), int(of.numel() - 1), int(eos_id))
    return args, keep


def _apply_mask(logits, trans, accept, live, num_symbols, dead, offsets, symbols, eos_id,
                states, neg_inf):
    args, keep = _dfa(trans, accept, live, num_symbols, dead, offsets, symbols, eos_id)
    V = args[8]
    if logits.dim() != 2 or logits.shape[1] != V:
        raise RuntimeError("bpdecode: logits must be [batch, vocab]")
    code = _check_logits(logits, V)
    st = _c(states, torch.int32, "states")
    if st.numel() != logits.shape[0]:
        raise RuntimeError("bpdecode: one state per logits row")
    L = _capi.lib()
    L.check(L.bpd_walk_apply_mask(logits.data_ptr(), code, logits.stride(0), int(st.numel()),
                                  *args, st.data_ptr(), float(neg_inf), _stream(logits)))
    return logits


def _compute_mask(trans, accept, live, num_symbols, dead, offsets, symbols, eos_id, states):
    args, keep = _dfa(trans, accept, live, num_symbols, dead, offsets, symbols, eos_id)
    st = _c(states, torch.int32, "states")
    out = torch.empty((int(st.numel()), (args[8] + 31) // 32), dtype=torch.int32,
                      device=st.device)
    L = _capi.lib()
    L.check(L.bpd_walk_mask_bits(*args, st.data_ptr(), int(st.numel()), out.data_ptr(),
                                 _stream(out)))
    return out


def _advance_state(trans, accept, live, num_symbols, dead, offsets, symbols, eos_id, states,
                   token_ids):
    args, keep = _dfa(trans, accept, live, num_symbols, dead, offsets, symbols, eos_id)
    st = _c(states, torch.int32, "states")
    if token_ids.dtype != torch.int32:
        raise RuntimeError("bpdecode: states / token_ids must be int32")
    tk = _tokens(token_ids, int(st.numel()), st.device)
    out = torch.empty(int(st.numel()), dtype=torch.int32, device=st.device)
    L = _capi.lib()
    L.check(L.bpd_walk_advance(*args, st.data_ptr(), tk.data_ptr(), 0, int(st.numel()),
                               out.data_ptr(), _stream(out)))
    return out


def _build_reachability(trans, accept, num_symbols):
    """Host-only, like the reference: live[s] = an accepting state is reachable."""
    if trans.is_cuda:
        raise RuntimeError("build_reachability is host-only (run it once at compile time)")
    tr = trans.contiguous().numpy().astype(np.int64)
    ac = accept.contiguous().numpy().astype(bool)
    S, M = ac.size, int(num_symbols)
    preds: list[list[int]] = [[] for _ in range(S)]
    for s in range(S):
        for t in tr[s * M:(s + 1) * M]:
            if 0 <= t < S:
                preds[int(t)].append(s)
    live = ac.astype(np.uint8)
    work = [int(s) for s in np.nonzero(ac)[0]]
    while work:
        for p in preds[work.pop()]:
            if not live[p]:
                live[p] = 1
                work.append(p)
    return torch.from_numpy(live)


def _grammar(accept, live, edge_offsets, edge_kind, edge_lo, edge_hi, edge_dst, edge_callee,
             root_start, root_accept, tok_offsets=None, tok_bytes=None, eos_id=-1):
    keep = [_c(accept, torch.uint8, "accept"), _c(live, torch.uint8, "live"),
            _c(edge_offsets, torch.int32, "edge_offsets")]
    dev = keep[0].device
    for t, name in ((edge_kind, "edge_kind"), (edge_lo, "edge_lo"), (edge_hi, "edge_hi"),
                    (edge_dst, "edge_dst"), (edge_callee, "edge_callee")):
        x = _c(t, torch.int32, name)
        keep.append(x if x.numel() else torch.zeros(1, dtype=torch.int32, device=dev))
    if tok_offsets is None:  # pda_init: no vocabulary needed
        tok_offsets = torch.zeros(2, dtype=torch.int32, device=dev)
        tok_bytes = torch.zeros(1, dtype=torch.uint8, device=dev)
    to = _c(tok_offsets, torch.int32, "tok_offsets")
    tb = _c(tok_bytes, torch.uint8, "tok_bytes")
    if tb.numel() == 0:
        tb = torch.zeros(1, dtype=torch.uint8, device=dev)
    keep += [to, tb]
    g = _capi.PdaGrammar(
        int(keep[0].numel()), int(edge_kind.numel()), int(root_start), int(root_accept),
        *(k.data_ptr() for k in keep[:8]), int(to.numel() - 1), int(eos_id), to.data_ptr(),
        tb.data_ptr())
    return g, keep


def _check_configs(configs):
    if configs.dtype != torch.int32:
        raise RuntimeError("configs must be int32")
    if configs.dim() != 2 or configs.shape[1] != PDA_CONFIG_FLAT:
        raise RuntimeError(f"configs must be [batch, {PDA_CONFIG_FLAT}]")
    if not configs.is_contiguous():
        raise RuntimeError("configs must be contiguous")


def _pda_init(accept, live, edge_offsets, edge_kind, edge_lo, edge_hi, edge_dst, edge_callee,
              root_start, root_accept):
    g, keep = _grammar(accept, live, edge_offsets, edge_kind, edge_lo, edge_hi, edge_dst,
                       edge_callee, root_start, root_accept)
    out = torch.empty(PDA_CONFIG_FLAT, dtype=torch.int32, device=keep[0].device)
    L = _capi.lib()
    L.check(L.bpd_pda_init(C.byref(g), out.data_ptr(), _stream(out)))
    return out


def _pda_apply_mask(logits, accept, live, edge_offsets, edge_kind, edge_lo, edge_hi, edge_dst,
                    edge_callee, root_start, root_accept, tok_offsets, tok_bytes, eos_id, configs,
                    neg_inf):
    g, keep = _grammar(accept, live, edge_offsets, edge_kind, edge_lo, edge_hi, edge_dst,
                       edge_callee, root_start, root_accept, tok_offsets, tok_bytes, eos_id)
    _check_configs(configs)
    B = int(logits.shape[0])
    if configs.shape[0] != B:
        raise RuntimeError("one config-set per logits row")
    code = _check_logits(logits, g.vocab_size)
    L = _capi.lib()
    ws = torch.empty(L.bpd_pda_workspace_bytes(B, g.vocab_size), dtype=torch.uint8,
                     device=logits.device)
    L.check(L.bpd_pda_apply_mask(C.byref(g), logits.data_ptr(), code, logits.stride(0),
                                 configs.data_ptr(), None, None, B, None, 0, ws.data_ptr(),
                                 float(neg_inf), _stream(logits)))
    return logits


def _pda_advance_state(configs, accept, live, edge_offsets, edge_kind, edge_lo, edge_hi,
                       edge_dst, edge_callee, root_start, root_accept, tok_offsets, tok_bytes,
                       eos_id, token_ids):
    g, keep = _grammar(accept, live, edge_offsets, edge_kind, edge_lo, edge_hi, edge_dst,
                       edge_callee, root_start, root_accept, tok_offsets, tok_bytes, eos_id)
    _check_configs(configs)
    B = int(configs.shape[0])
    if token_ids.dtype != torch.int32 or token_ids.numel() != B:
        raise RuntimeError("token_ids must be int32, one per config-set")
    tk = _tokens(token_ids, B, configs.device)
    ok = torch.empty(B, dtype=torch.uint8, device=configs.device)
    L = _capi.lib()
    L.check(L.bpd_pda_advance(C.byref(g), configs.data_ptr(), None, B, tk.data_ptr(), 0,
                              ok.data_ptr(), None, None, _stream(ok)))
    return ok


_IMPLS = {
    "apply_mask_": _apply_mask, "compute_mask": _compute_mask, "advance_state": _advance_state,
    "pda_init": _pda_init, "pda_apply_mask_": _pda_apply_mask,
    "pda_advance_state": _pda_advance_state,
}


def register() -> torch.library.Library:
    """Define the ``bpdecode`` namespace's ops (idempotent)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    try:
        lib = torch.library.Library("bpdecode", "DEF")
    except RuntimeError as exc:  # the reference's extension already owns the namespace
        raise ImportError(
            "torch.ops.bpdecode is already registered (bpdecode's own extension is loaded); "
            "load one implementation per process") from exc
    for schema in SCHEMAS.values():
        lib.define(schema)
    for name, fn in _IMPLS.items():
        lib.impl(name, fn, "CUDA")
    lib.impl("build_reachability", _build_reachability, "CPU")
    _LIB = lib
    return lib


register()
