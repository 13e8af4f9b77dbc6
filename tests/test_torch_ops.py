"""torch.ops.bpdecode.* registration (CPU side: schemas, the host-only
build_reachability op, and loud failure for CPU tensors on device ops)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_npz, small_cases, small_dfa

SMALL = golden_npz("small.npz")


def test_schemas_match_the_reference() -> None:
    import bpdecode_b200.torch_ops as T

    for name, schema in T.SCHEMAS.items():
        op = getattr(torch.ops.bpdecode, name)
        assert str(op.default._schema) == "bpdecode::" + schema, name


@pytest.mark.parametrize("vname,pi", small_cases()[::4])
def test_build_reachability_matches_reference_tables(vname: str, pi: int) -> None:
    import bpdecode_b200.torch_ops  # noqa: F401

    dfa = small_dfa(SMALL, vname, pi)
    live = torch.ops.bpdecode.build_reachability(
        torch.from_numpy(dfa["trans"]), torch.from_numpy(dfa["accept"]), dfa["num_symbols"])
    assert np.array_equal(live.numpy(), dfa["live"])


def test_device_ops_reject_cpu_tensors() -> None:
    import bpdecode_b200.torch_ops  # noqa: F401

    z = torch.zeros(1, 4)
    i = torch.zeros(4, dtype=torch.int32)
    u = torch.zeros(1, dtype=torch.uint8)
    with pytest.raises((NotImplementedError, RuntimeError)):
        torch.ops.bpdecode.apply_mask_(z, i, u, u, 1, 0, torch.zeros(5, dtype=torch.int32), i, 3,
                                       torch.zeros(1, dtype=torch.int32), float("-inf"))
