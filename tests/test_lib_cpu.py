"""The C-ABI library without a GPU: it loads, exports every entry point that
include/iam.h declares, and rejects bad arguments before touching the device."""
import os
import re

import pytest

import iam_b200 as I

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared():
    text = open(os.path.join(ROOT, "include", "iam.h")).read()
    return set(re.findall(r"\b(iam_[a-z0-9_]+)\s*\(", text))


def test_header_and_binding_agree():
    assert declared() == set(I.exported_symbols())


def test_library_exports_every_declared_symbol():
    lib = I.lib()
    for name in declared():
        assert hasattr(lib, name), name


def test_argument_validation_without_gpu():
    with pytest.raises(I.IamError) as e:
        I.qmm_affine4(0, 0, 0, 0, 0, 1, 16, 64, 64)
    assert e.value.status == I.IAM_EINVAL
    with pytest.raises(I.IamError):
        I.sdpa_decode_append(0, 0, 0, 0, 0, 0, 1, 0, 24, 4, 256, 16)
    with pytest.raises(I.IamError):
        I.gated_delta_step(16, 16, 16, 16, 16, 16, 16, 48, 16, 64, 128, 1)


def test_dims_defaults_are_qwen35_27b():
    d = I.Dims.qwen35_27b()
    assert (d.hidden, d.intermediate, d.vocab, d.n_layers) == (5120, 17408, 248320, 64)
    assert (d.gdn_k_heads, d.gdn_v_heads, d.n_heads, d.n_kv_heads, d.head_dim) == (16, 48, 24, 4, 256)
    assert abs(d.rope_theta - 1e7) < 1 and d.rotary_dim == 64
    assert d.max_seqs == 1


def test_sequence_slots_are_validated():
    """max_seqs (the multi-sequence verify's slots) must lie in 1..max_rows;
    checked by the host-only shard planner, no GPU involved."""
    for bad in (0, 129):
        d = I.Dims.qwen35_27b(max_rows=128, max_seqs=bad)
        with pytest.raises(I.IamError) as err:
            I.tp_shard_of(d, 0, 1)
        assert err.value.status == I.IAM_EINVAL and "max_seqs" in str(err.value)
    I.tp_shard_of(I.Dims.qwen35_27b(max_rows=512, max_seqs=64), 0, 8)
