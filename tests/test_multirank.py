"""The multi-GPU path's host logic on CPU: the row-sharding rule of every multi-GPU forward (jc_shard_rows),
and bench.py's per-rank batch split and max-over-ranks timing across two gloo ranks on 127.0.0.1."""

import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import jitcast_b200
from jitcast_b200 import _lib

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

import bench  # noqa: E402


def random_series(rng, rows):
    """group_start / group_end of contiguous series of random lengths (1-6 rows)."""
    gs, ge, i = np.empty(rows, np.int32), np.empty(rows, np.int32), 0
    while i < rows:
        e = min(rows, i + int(rng.integers(1, 7)))
        gs[i:e], ge[i:e] = i, e
        i = e
    return gs, ge


@pytest.mark.parametrize("rows,parts", [(0, 2), (1, 8), (7, 2), (50, 3), (203, 8), (64, 64)])
def test_shard_rows_keeps_series_whole(rows, parts):
    rng = np.random.default_rng(rows * 31 + parts)
    gs, ge = random_series(rng, rows)
    cuts = jitcast_b200.shard_rows(gs, ge, parts)
    assert len(cuts) == parts + 1 and cuts[0] == 0 and cuts[-1] == rows
    assert np.all(np.diff(cuts) >= 0)
    for p in range(1, parts):
        c = int(cuts[p])
        assert c == rows or gs[c] == c  # on a series boundary
        # the even split point (not before the previous cut), moved forward to the end of the series holding it
        t = max(rows * p // parts, int(cuts[p - 1]))
        assert c == (t if t >= rows or gs[t] == t else ge[t])


def test_shard_rows_rejects_split_series():
    gs = np.array([0, 0, 2, 0], np.int32)
    ge = np.array([2, 2, 3, 2], np.int32)
    with pytest.raises(jitcast_b200.JcArgumentError, match="contiguous"):
        jitcast_b200.shard_rows(gs, ge, 2)
    assert _lib.lib().jc_shard_rows(4, gs.ctypes.data, ge.ctypes.data, 0, None) == _lib.ERR_INVALID_ARG


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_rank_chunks_partition_the_batch(world):
    whole = bench.rank_chunks(65536, 8192, 1, 0)
    parts = [ch for r in range(world) for ch in bench.rank_chunks(65536, 8192, world, r)]
    assert parts == whole  # the same chunks, hence the same seeded series, for every N


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_gather_the_single_rank_result(tmp_path):
    import multirank_worker as mw
    from jitcast_b200 import timestral as ts
    from oracle import timestral as ots

    out = tmp_path / "ranks.npz"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", str(HERE / "multirank_worker.py"), str(out)]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    got = np.load(out)
    assert float(got["slowest"]) == 2.0  # max over the ranks' 1.0 and 2.0
    c = mw.tiny_config()
    model = ots.Model(c, ts.random_checkpoint(c, seed=3))
    whole = bench.rank_chunks(mw.SERIES, mw.CHUNK, 1, 0)
    assert sorted(k for k in got.files if k.startswith("chunk_")) == sorted(f"chunk_{c0}" for c0, _ in whole)
    for c0, n in whole:
        np.testing.assert_array_equal(got[f"chunk_{c0}"], mw.chunk_forecast(model, c0, n))
