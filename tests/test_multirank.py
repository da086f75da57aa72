"""The N>1 host path of bench.py on CPU: two gloo ranks on 127.0.0.1.

One process per GPU in the real job; here each rank is a CPU process running
the same host logic: per-rank inputs (utterances shard by request, no
collective on the data path), the max-over-ranks time, the whole-job
throughput, and the reference arm that only rank 0 runs."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import bench
    dist = bench.init_process_group(world, rank, "gloo")
    try:
        x = bench.synthetic_logmels(2, 8, 16, bench.rank_input_seed(rank))
        # a rank-dependent device time; the job time is the slowest rank's
        ms = 10.0 + 20.0 * rank
        job_ms = bench.max_over_ranks(ms, dist, "cpu")
        value, tok_s = bench.job_throughput(world, clips=64, steps=3, tokens=128, ms=job_ms)

        class A:
            warmup, steps, tokens, gpus = 0, 1, 1, world
        printed = rank != 0  # rank 0 would run the CPU reference; only check that the others do nothing
        if rank != 0:
            import io, contextlib
            buf = io.StringIO()
            with contextlib.redirect_stdout(buf):
                bench.run_reference(A, rank)
            printed = buf.getvalue() == ""
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), x=x, job_ms=job_ms, value=value, tok_s=tok_s,
                 ref_silent=printed)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_ranks_gloo(tmp_path):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.spawn(_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    r = [np.load(tmp_path / f"r{i}.npz") for i in range(2)]
    # each rank decodes different utterances
    assert not np.array_equal(r[0]["x"], r[1]["x"])
    # max over ranks, identical on every rank
    assert float(r[0]["job_ms"]) == float(r[1]["job_ms"]) == 30.0
    # whole-job throughput: both ranks' clips over the slowest rank's time
    assert float(r[0]["value"]) == pytest.approx(2 * 64 * 30.0 * 3 / 0.030)
    assert float(r[0]["tok_s"]) == pytest.approx(2 * 64 * 128 * 3 / 0.030)
    # the reference arm prints from rank 0 only
    assert bool(r[1]["ref_silent"])


def test_throughput_workload_shards():
    """configs[4] workload per rank: seeded, distinct across ranks, within the
    config's ranges (clips 5-30 s, decode lengths 32-224)."""
    import bench
    a, sa = bench.throughput_utterances(256, 0, 64)
    b, sb = bench.throughput_utterances(256, 0, 64)
    c, _ = bench.throughput_utterances(256, 1, 64)
    assert [(u.n_samples, u.n_new_tokens) for u in a] == [(u.n_samples, u.n_new_tokens) for u in b] and sa == sb
    assert [(u.n_samples, u.n_new_tokens) for u in a] != [(u.n_samples, u.n_new_tokens) for u in c]
    assert all(5 * 16000 <= u.n_samples <= 30 * 16000 and 32 <= u.n_new_tokens <= 224 for u in a)
    assert all(u.pcm_index == i % 64 for i, u in enumerate(a))
    assert abs(sa - sum(u.n_samples for u in a) / 16000) < 256 / 16000 + 1e-6


def _dying_rank_main(rank, world, port, out_dir):
    import sys
    import time
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import bench
    dist = bench.init_process_group(world, rank, "gloo", timeout_s=3.0)
    dist.barrier()  # both ranks took part in the first step
    if rank == 1:
        os._exit(0)  # the shard dies between steps, with nothing in flight
    t0 = time.time()
    err = ""
    try:
        bench.max_over_ranks(10.0, dist, "cpu")  # the next step's max-over-ranks time
    except Exception as e:  # the collective fails instead of waiting forever
        err = type(e).__name__
    waited = time.time() - t0
    # the dead rank's utterances are a pure function of its rank: a surviving rank re-queues them
    utts, _ = bench.throughput_utterances(64, 1, 16)
    np.savez(os.path.join(out_dir, "survivor.npz"), err=err, waited=waited,
             requeued=np.array([(u.n_samples, u.n_new_tokens) for u in utts]))
    os._exit(0)


def test_rank_death_is_detected_and_its_shard_requeued(tmp_path):
    """A rank that leaves between steps (no kernel or collective in flight):
    the survivor's next collective raises within the process-group timeout
    instead of hanging, and the dead rank's share of utterances, seeded by its
    rank, is rebuilt on the survivor unchanged."""
    import torch.multiprocessing as mp
    import bench
    port = _free_port()
    ctx = mp.start_processes(_dying_rank_main, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    for p in ctx.processes:
        p.join(60)
        assert not p.is_alive()
    r = np.load(tmp_path / "survivor.npz")
    assert str(r["err"]) != ""
    assert float(r["waited"]) < 30.0
    want, _ = bench.throughput_utterances(64, 1, 16)
    assert np.array_equal(r["requeued"], np.array([(u.n_samples, u.n_new_tokens) for u in want]))
