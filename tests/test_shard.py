"""Multi-rank host logic on CPU: utterance placement over ranks and the
max-over-ranks timing reduction, run as world-size-2 gloo process groups.
A rank that fails before the timing collective is detected by the surviving
rank through a short process-group timeout (no GPU involved)."""
import datetime
import multiprocessing as mp
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def _shard():
    import __graft_entry__ as ge
    ge.load_package()
    import importlib
    return importlib.import_module("qwen_asr_b200.shard")


@pytest.mark.parametrize("n,world", [(64, 1), (64, 2), (64, 8), (7, 3), (3, 8), (0, 4)])
def test_shard_range_partitions(n, world):
    shard = _shard()
    seen = []
    sizes = []
    for r in range(world):
        first, cnt = shard.shard_range(n, world, r)
        seen.extend(range(first, first + cnt))
        sizes.append(cnt)
    assert seen == list(range(n))          # contiguous, disjoint, complete, in rank order
    assert max(sizes) - min(sizes) <= 1


def test_shard_range_rejects_bad_rank():
    shard = _shard()
    with pytest.raises(ValueError):
        shard.shard_range(8, 2, 2)
    with pytest.raises(ValueError):
        shard.shard_range(8, 0, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    try:
        import torch.distributed as dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=5))
        shard = _shard()
        if mode == "fail" and rank == 1:
            q.put((rank, "raised"))
            q.close()
            q.join_thread()      # flush before the hard exit
            os._exit(3)          # leaves between steps, before the timing collective
        first, cnt = shard.shard_range(64, world, rank)
        vals = shard.max_over_ranks([10.0 + rank, 5.0 - rank, float(cnt)])
        sums = shard.sum_over_ranks([float(cnt), 1.0])
        dist.barrier()
        q.put((rank, ("ok", first, cnt, vals + sums)))
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, ("error", type(e).__name__)))


def _run(world, mode, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = {}
    for _ in range(world):
        r, v = q.get(timeout=timeout)
        out[r] = v
    for p in ps:
        p.join(timeout=timeout)
        if p.is_alive():
            p.kill()
    return out, [p.exitcode for p in ps]


def test_gloo_two_ranks_max_and_placement():
    out, codes = _run(2, "ok")
    assert codes == [0, 0]
    for r in range(2):
        tag, first, cnt, vals = out[r]
        assert tag == "ok" and (first, cnt) == (32 * r, 32)
        assert vals == [11.0, 5.0, 32.0, 64.0, 2.0]   # the slowest rank's time; whole-job counts


def test_gloo_rank_failure_detected_by_survivor():
    out, codes = _run(2, "fail")
    assert out[1] == "raised" and codes[1] == 3
    assert out[0][0] == "error"            # collective ended with an error, no hang
