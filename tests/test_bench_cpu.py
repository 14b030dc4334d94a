"""Host logic of bench.py that needs no GPU: the exposed-time accounting of
--trace-step (kernel records as CUPTI reports them, overlapping under
programmatic dependent launch)."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def ev(name, ts, dur, grid=None):
    return {"name": name, "ts": ts, "dur": dur, "args": {"grid": grid} if grid else {}}


def test_exposed_time_sums_to_the_span():
    # a matmul, a GDN kernel launched early that ends after it, a matmul
    # fully hidden under the GDN kernel, a gap, then the norm
    events = [
        ev("void iam::qmm_tc_kernel<32>(...)", 0.0, 10.0, [272, 1, 1]),
        ev("void iam::gdn_fused_kernel<2, false, false>(...)", 6.0, 8.0, [96, 1, 1]),
        ev("void iam::qmm_tc_kernel<32>(...)", 7.0, 5.0, [40, 1, 3]),
        ev("void iam::rms_norm_row_kernel<20>(...)", 20.0, 2.0, [32, 1, 1]),
    ]
    kinds, span = bench.exposed_by_kind(events)
    assert span == 22.0
    assert kinds["qmm_tc gate_up"] == [1, 10.0, 10.0]
    assert kinds["gdn_fused"] == [1, 8.0, 4.0]          # 6..14, of which 10..14 extend the span
    assert kinds["qmm_tc out_proj|o_proj|down"] == [1, 5.0, 0.0]
    assert kinds["rms_norm"] == [1, 2.0, 2.0]           # the gap 14..20 belongs to no kernel
    assert sum(r[2] for r in kinds.values()) + 6.0 == span


def test_kernel_kind_names():
    assert bench.kernel_kind("void iam::(anonymous namespace)::qmm_gemv_kernel<1, 2>(...)", [1940, 1, 1]) == \
        "qmm_gemv lm_head"
    assert bench.kernel_kind("void iam::attn_decode_tc_kernel<false>(...)", [32, 4, 3]) == "attn_decode_tc"
    assert bench.kernel_kind("void iam::attn_decode_kernel<false>(...)", None) == "attn_decode"
    assert bench.kernel_kind("some_library_kernel", None) == "some_library_kernel"
