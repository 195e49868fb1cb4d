"""bench.py's host-side accounting, checked without a GPU: which chains have the first net's input
pack written by the colour pre pass (one launch a frame fewer in `gpu_launches`), and the chain
FLOP count the roofline's frame figures divide by, against the architectures' closed forms."""
import os
import sys

import ajib

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def test_fused_pack_counts_plain_and_unshuffled_heads():
    # a head reading the NCHW RGB input, plain (Compact, SPAN) or 2x pixel-unshuffled (SPANF3)
    assert bench.fused_pack([ajib.compact_plan(1, c=16, body=1)]) == 1
    assert bench.fused_pack([ajib.span_plan(1, c=16, blocks=1)]) == 1
    assert bench.fused_pack([ajib.spanf3_plan(1, c=16, blocks=1)]) == 1


def test_fused_pack_follows_the_first_nets_head_only():
    plan = ajib.compact_plan(2, c=16, body=1)
    plan["steps"][0]["in_"] = ajib.IN_NHWC  # a head reading a strip-chunked map: nothing to pack
    assert bench.fused_pack([plan]) == 0
    assert bench.fused_pack([plan, ajib.compact_plan(3, c=16, body=1)]) == 0
    assert bench.fused_pack([ajib.compact_plan(3, c=16, body=1), plan]) == 1


def test_chain_flops_spanf3_b5f48_1080p():
    """SPANF3 b5f48 at 1920x1080: convs at 960x540 after the 2x unshuffle. Per conv pixel: head
    3x3 12->48, five blocks of three 3x3 48->48 convs plus the tanh gate's 1x1 48->48, the concat
    1x1 192->48, the tail 3x3 48->48; 2 FLOPs a multiply-add."""
    per_px = 2 * 9 * 12 * 48 + 5 * (3 * 2 * 9 * 48 * 48 + 2 * 48 * 48) + 2 * 192 * 48 + 2 * 9 * 48 * 48
    assert per_px == 715392
    got = bench.chain_flops([ajib.spanf3_plan(1, c=48, blocks=5)], 1920, 1080)
    assert got == per_px * 960 * 540


def test_chain_flops_two_compact_chain():
    """Two Compact 2x nets chained (960x540 -> 1920x1080 -> 3840x2160): the second runs at the first's
    output size. Compact 64 x 16 body: head 3->64, 16 body 64->64, tail 64->12, all 3x3."""
    per_px = 2 * 9 * (3 * 64 + 16 * 64 * 64 + 64 * 12)
    plans = [ajib.compact_plan(4, c=64, body=16), ajib.compact_plan(5, c=64, body=16)]
    assert bench.chain_flops(plans, 960, 540) == per_px * (960 * 540 + 1920 * 1080)
