"""The ranks' rendezvous (tpcuda.store) on CPU: several processes exchange the
NCCL unique id, meet at barriers, take a max over ranks and gather arrays
through one shared directory; a rank that never arrives makes the others raise
TimeoutError instead of hanging; the directory is gone after close()."""
import multiprocessing as mp
import os
import time

import numpy as np
import pytest

from tpcuda.store import FileStore, default_dir


def _rank_main(rank, world, path, q):
    try:
        st = FileStore(rank, world, path, timeout_s=30)
        uid = st.broadcast_bytes(os.urandom(128) if rank == 0 else None, "nccl-unique-id")
        st.barrier()
        mx = st.max(float(rank * 10 + 1))
        arrs = st.all_gather_array(np.arange(4, dtype=np.float32) + rank)
        objs = st.all_gather_obj({"rank": rank})
        st.barrier()
        st.close()
        q.put((rank, uid.hex(), mx, [a.tolist() for a in arrs], objs))
    except Exception as e:  # reported to the parent
        q.put((rank, "error", repr(e), None, None))


@pytest.mark.parametrize("world", [2, 3])
def test_ranks_share_id_barrier_max_gather(tmp_path, world):
    path = str(tmp_path / "store")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_main, args=(r, world, path, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[1] != "error" for r in res), res
    assert len({r[1] for r in res}) == 1 and len(res[0][1]) == 256  # one 128-byte id on every rank
    assert all(r[2] == float((world - 1) * 10 + 1) for r in res)
    for r in res:
        assert r[3] == [[k, k + 1, k + 2, k + 3] for k in range(world)]
        assert r[4] == [{"rank": k} for k in range(world)]
    assert not os.path.exists(path)


def test_missing_rank_times_out(tmp_path):
    st = FileStore(0, 2, str(tmp_path / "s"), timeout_s=0.5)
    t0 = time.monotonic()
    with pytest.raises(TimeoutError):
        st.barrier()
    assert time.monotonic() - t0 < 5


def test_default_dir_is_per_launch(monkeypatch):
    monkeypatch.delenv("TPCUDA_STORE_DIR", raising=False)
    monkeypatch.setenv("MASTER_PORT", "29511")
    d = default_dir()
    assert "29511" in d and str(os.getppid()) in d
    monkeypatch.setenv("TPCUDA_STORE_DIR", "/tmp/x-store")
    assert default_dir() == "/tmp/x-store"


def _leaver(rank, world, path, q):
    st = FileStore(rank, world, path, timeout_s=30)
    st.barrier()
    if rank == 1:
        st.leave()
        q.put((rank, []))
        return
    import time as _t
    t0 = _t.monotonic()
    while not st.departed() and _t.monotonic() - t0 < 20:
        _t.sleep(0.01)
    q.put((rank, st.departed()))


def test_departed_rank_is_seen_before_the_next_step(tmp_path):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    path = str(tmp_path / "s")
    ps = [ctx.Process(target=_leaver, args=(r, 2, path, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=60) for _ in range(2))
    for p in ps:
        p.join(timeout=30)
    assert res[0] == [1] and res[1] == []
