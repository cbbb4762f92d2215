"""Failure detection on the host (gloo ranks on CPU; no GPU is faulted): silent and failing ranks
are reported by the heartbeat, a rank that never joins ends the rendezvous with an error, damaged
checkpoints are refused, and recorded device-wait timeouts surface as exceptions."""
import datetime
import os
import socket
import time

import pytest
import torch


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, scenario, q):
    import torch.distributed as dist

    from trida_stack_b200.parallel.health import Heartbeat, RankFailure
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    hb = Heartbeat(interval=0.05, timeout=1.0).start()
    t0 = time.time()
    if rank == 1:
        if scenario == "fail":
            hb.fail("out of memory in step 3")
            time.sleep(2.0)
        elif scenario == "silent":
            hb.stop()                       # stops publishing: a hung rank
            time.sleep(4.0)
        elif scenario == "exit":
            os._exit(0)                     # leaves without saying goodbye
        hb.stop()
        q.put((rank, "done", None))
        q.close()
        q.join_thread()
        os._exit(0)
    got = None
    while time.time() - t0 < 8.0:
        try:
            hb.check()
        except RankFailure as e:
            got = (sorted(e.failed), str(e), round(time.time() - t0, 2))
            break
        time.sleep(0.05)
    hb.stop()
    q.put((rank, "detected" if got else "missed", got))
    q.close()
    q.join_thread()                         # flush the result before leaving
    os._exit(0)                             # rank 1 may be gone: skip the collective teardown


@pytest.mark.parametrize("scenario", ["fail", "silent", "exit"])
def test_heartbeat_reports_failed_silent_and_departed_ranks(scenario):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, scenario, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    deadline = time.time() + 60
    while len(res) < (1 if scenario == "exit" else 2) and time.time() < deadline:
        try:
            r, status, info = q.get(timeout=1)
            res[r] = (status, info)
        except Exception:
            pass
    for p in procs:
        p.join(timeout=20)
        if p.is_alive():
            p.kill()
    status, info = res[0]
    assert status == "detected", res
    failed, msg, after = info
    assert failed == [1]
    if scenario == "fail":
        assert "out of memory" in msg and after < 1.0      # told, not timed out
    else:
        assert after < 5.0


def _lonely(port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=2))
        q.put(("joined", time.time() - t0))
    except Exception as e:
        q.put((type(e).__name__, time.time() - t0))


def test_rank_that_never_joins_ends_the_rendezvous():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_port(), q))
    p.start()
    what, dt = q.get(timeout=60)
    p.join(timeout=10)
    assert what != "joined" and dt < 30


def test_damaged_checkpoint_is_refused(tmp_path):
    from trida_stack_b200.checkpoint import CheckpointCorrupt, verify_manifest, write_manifest
    d = tmp_path / "step_10"
    (d / "train_state").mkdir(parents=True)
    (d / "model.safetensors").write_bytes(os.urandom(4096))
    (d / "train_state" / "__0_0.distcp").write_bytes(os.urandom(1000))
    (d / "config.json").write_text("{}")
    write_manifest(str(d))
    assert verify_manifest(str(d))
    raw = bytearray((d / "model.safetensors").read_bytes())
    raw[100] ^= 0xFF
    (d / "model.safetensors").write_bytes(bytes(raw))
    with pytest.raises(CheckpointCorrupt, match="model.safetensors"):
        verify_manifest(str(d))
    raw[100] ^= 0xFF
    (d / "model.safetensors").write_bytes(bytes(raw[:2048]))            # truncated
    with pytest.raises(CheckpointCorrupt, match="bytes"):
        verify_manifest(str(d))
    (d / "model.safetensors").write_bytes(bytes(raw))
    os.remove(d / "train_state" / "__0_0.distcp")                      # a lost optimizer shard
    with pytest.raises(CheckpointCorrupt, match="missing"):
        verify_manifest(str(d))


def test_recorded_device_timeout_raises(monkeypatch):
    from trida_stack_b200.ops import blocks
    from trida_stack_b200.parallel.health import DeviceWaitTimeout, check_device

    class FakeExt:
        @staticmethod
        def gemm_error():
            return 104                       # an mbarrier wait of the GEMM gave up

    monkeypatch.setattr(blocks, "ext", lambda: FakeExt())
    monkeypatch.setitem(blocks._ERR_WORDS, "test", torch.zeros(1, dtype=torch.int32))
    with pytest.raises(DeviceWaitTimeout, match="104"):
        check_device()
