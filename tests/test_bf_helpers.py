"""The reference's public launch heuristics, kept in gpu_algo_b200.bf, pick the same
blocks as the reference's own functions (tests/golden/block_choices.json, generated
from them by tests/golden/make_block_choices.py)."""
import json
import os

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _cases():
    with open(os.path.join(GOLDEN, "block_choices.json")) as f:
        return json.load(f)


def test_choose_block_matches_reference():
    from gpu_algo_b200.bf.fp32 import choose_block
    cases = _cases()["choose_block"]
    assert len(cases) > 100
    for k, d, block in cases:
        assert choose_block(k, d) == block, (k, d)


def test_choose_qgroup_block_matches_reference():
    from gpu_algo_b200.bf.fp32_qgroup import choose_qgroup_block
    cases = _cases()["choose_qgroup_block"]
    assert len(cases) > 500
    for k, d, qpb, block in cases:
        assert choose_qgroup_block(k, d, qpb) == block, (k, d, qpb)
