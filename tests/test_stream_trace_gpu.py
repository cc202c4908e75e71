"""The stream decode's per-warp timeline (``bench.py --op trace``) on a B200.

The trace build of the library stamps %globaltimer in the stream and warp-fixup
kernels; the op runs the headline layer-steps (KV write + scheduled decode) in
a CUDA graph and prints per-launch figures.  The run goes in a child process:
it loads ``libmvb200_trace.so`` in place of the product library.  The checks
are the order of events every launch must show.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.gpu
def test_stream_trace_orders_the_events():
    res = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--op", "trace", "--config", "2",
                          "--layers", "3"], capture_output=True, text=True, timeout=600, cwd=REPO)
    assert res.returncode == 0, res.stderr[-3000:]
    lines = [json.loads(x) for x in res.stdout.splitlines() if x.startswith("{")]
    head, rows = lines[0], lines[1:]
    assert head["op"] == "trace" and head["layers"] == 3 and head["plan"]["variant"] == "stream"
    assert len(rows) == 3
    for r in rows:
        assert r["warps_with_tiles"] > 0 and r["stream_warps"] >= r["warps_with_tiles"]
        assert 0.0 <= r["entry_p50_us"] <= r["first_issue_p50_us"] <= r["first_tile_us"][1]
        assert r["first_tile_us"][0] <= r["first_tile_us"][1] <= r["first_tile_us"][2]
        assert r["first_tile_us"][2] <= r["loop_end_us"][2] <= r["stream_end_max_us"]
        assert r["tile_interval_p50_us"] > 0.0
        # config 2 cuts units at warp-range boundaries: the fixup merges them after the stream warps
        assert r["fixup_warps"] > 0 and r["fixup_end_max_us"] >= r["fixup_wait_us"][1]
        # the fixup's wait returns only after every stream warp has ended (one global timer)
        assert r["fixup_wait_us"][0] >= r["stream_end_max_us"] - 0.5
        assert r["stream_end_max_us"] < 1000.0
    assert all(r["start_after_previous_us"] is not None for r in rows[1:])
