"""Host logic of tensor parallelism on CPU (gloo, world size 2): every rank
receives rank 0's unique id; a rank whose peer never reaches the handshake
gives up with an error after the group's timeout instead of waiting for
good; and the sharding rule refuses shapes whose slices do not fall on
32-element blocks."""
import datetime
import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, out):
    import torch.distributed as dist
    from catseye_b200.llm import tp_share_id
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = tp_share_id(make_id=lambda: bytes(range(128)) if rank == 0 else b"wrong")
        out.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_unique_id_reaches_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0] == res[1] == bytes(range(128))


def _absent_peer_rank(rank, world, port, out, done):
    """Rank 1 joins the group and then never takes part in the handshake (a
    rank stuck or lost before it); rank 0 runs the handshake and reports how
    it ended."""
    import torch.distributed as dist
    from catseye_b200.llm import tp_share_id
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        # the rendezvous waits as long as the slowest process takes to start;
        # the handshake runs on a group of its own with a short timeout
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        group = dist.new_group(ranks=list(range(world)), timeout=datetime.timedelta(seconds=3))
    except Exception as e:
        out.put(("setup failed: " + repr(e), 0.0))
        _flush_exit(out)
    if rank == 0:
        t0 = time.monotonic()
        try:
            tp_share_id(group=group, make_id=lambda: bytes(128))
            out.put(("returned", time.monotonic() - t0))
        except Exception as e:   # the group's timeout: the handshake gives up
            out.put((type(e).__name__, time.monotonic() - t0))
    else:
        done.wait(120)   # alive but silent until rank 0 has its answer
    _flush_exit(out)     # no collective teardown with a peer that never answered


def _flush_exit(out):
    """Exit at once, after the queue's feeder thread has written what was put."""
    out.close()
    out.join_thread()
    os._exit(0)


def test_handshake_gives_up_when_a_peer_never_arrives():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_absent_peer_rank, args=(r, 2, port, q, done)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        how, waited = q.get(timeout=120)
    finally:
        done.set()
        for p in procs:
            p.join(timeout=60)
    assert not how.startswith("setup failed"), how
    assert how != "returned", "the handshake completed without its peer"
    assert waited < 60, waited


@pytest.mark.parametrize("dim,heads,kv,hidden,tp,ok", [
    (4096, 32, 32, 11008, 2, True), (4096, 32, 32, 11008, 8, True), (8192, 64, 8, 28672, 8, True),
    (288, 6, 6, 768, 2, False),      # 144 columns per rank: not a whole number of 32-blocks
    (512, 8, 2, 1376, 4, False),     # 2 kv heads cannot split 4 ways
    (4096, 32, 32, 11008, 3, False)])
def test_sharding_rule(dim, heads, kv, hidden, tp, ok):
    """The rule llm_alloc applies (C side) restated: heads, kv heads, hidden
    and vocab split evenly, every column slice a whole number of blocks."""
    vocab = 32000
    fits = (dim % heads == 0 and heads % kv == 0 and heads % tp == 0 and kv % tp == 0 and hidden % tp == 0
            and vocab % tp == 0 and (hidden // tp) % 32 == 0 and (dim // tp) % 32 == 0)
    assert fits == ok
