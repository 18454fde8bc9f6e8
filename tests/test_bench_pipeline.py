"""Copy groups of bench.py's e2e pipeline graph (CPU).

Every step of a captured pipeline must upload its own inputs and download its
own output exactly once inside the graph, the first kernel must wait for its
own upload only, and the compute stream must wait on the upload stream only a
few times (each wait costs that kernel its early start).
"""

import importlib.util
from pathlib import Path

import pytest

_spec = importlib.util.spec_from_file_location("bench", Path(__file__).resolve().parents[1] / "bench.py")
bench = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(bench)


@pytest.mark.parametrize("P", [1, 2, 3, 7, 8, 15, 16, 31, 32, 33, 64, 100])
def test_every_step_copied_once(P):
    up, down = bench.pipeline_groups(P)
    for groups in (up, down):
        steps = [k for a, b in groups for k in range(a, b)]
        assert steps == list(range(P))
        assert all(a < b for a, b in groups)
    assert up[0] == (0, 1)                      # the first kernel waits for its own inputs only
    assert down[-1] == (P - 1, P)               # one download after the last kernel
    assert len(up) <= 3 + (P - 1) // 32         # few waits on the uploads


def test_graph_sizes():
    up, down = bench.pipeline_groups(bench.E2E_GRAPH_STEPS)
    assert up == [(0, 1), (1, 7), (7, 31), (31, 64)]
    assert down[0] == (0, 7) and all(b - a <= 8 for a, b in down)
