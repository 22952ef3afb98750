"""Host-side failure detection (CPU, gloo): a rank that never joins a collective
ends the others' wait with an error within the process-group timeout, the way
the Ulysses runtime's short default timeout is meant to work."""
import multiprocessing
import os
import tempfile
import time
from datetime import timedelta

import torch
import torch.distributed as dist


def _rank(rank, rendezvous, q):
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=rendezvous, rank=rank, world_size=2,
                            timeout=timedelta(seconds=5))
    if rank == 1:
        # Leaves between steps, with nothing in flight, never joining the next collective.
        q.put(("left", 0.0))
        time.sleep(12)
        os._exit(0)
    t = torch.ones(4)
    t0 = time.monotonic()
    try:
        dist.all_reduce(t)
        q.put(("completed", time.monotonic() - t0))
    except Exception as e:  # gloo reports the timeout as an exception
        q.put(("error:" + type(e).__name__, time.monotonic() - t0))
    os._exit(0)


def test_missing_rank_times_out_with_error():
    ctx = multiprocessing.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d:
        procs = [ctx.Process(target=_rank, args=(r, "file://" + d + "/pg", q)) for r in range(2)]
        old = os.environ.get("CUDA_VISIBLE_DEVICES")
        os.environ["CUDA_VISIBLE_DEVICES"] = ""
        try:
            for p in procs:
                p.start()
        finally:
            if old is None:
                os.environ.pop("CUDA_VISIBLE_DEVICES", None)
            else:
                os.environ["CUDA_VISIBLE_DEVICES"] = old
        # Spawned ranks import torch cold, which can take a minute on a loaded host; the
        # bound under test is the in-rank time asserted below.
        results = [q.get(timeout=240) for _ in range(2)]
        for p in procs:
            p.join(30)
            if p.is_alive():
                p.terminate()
                p.join()
    outcome = dict(results)
    assert "left" in outcome
    errs = [k for k in outcome if k.startswith("error:")]
    assert errs, outcome
    assert outcome[errs[0]] < 30.0
