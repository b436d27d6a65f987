"""The sequence split's host orchestration on CPU: world-size 2 (and 3)
gloo process groups, each rank a SeqShard over its contiguous slice with
the oracle behind the ops signatures, exchanging candidates and partials
with real all-gathers.  Every rank's combined output must equal the
unsplit oracle step; a rank that leaves between steps must make each of
the others raise from its own next exchange, not hang."""

import os
import socket
import sys

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))

B, T_TOTAL, W, K, STEPS = 1, 96, 8, 16, 5
POS0 = 4 * T_TOTAL - 1 - STEPS - 2   # the last steps fill the last rows
MAX_SEQ = 4 * T_TOTAL + 16


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, Bn, fail_rank):
    sys.path[:0] = [os.path.dirname(HERE), os.path.join(os.path.dirname(HERE), "tt-deepseek-v4_b200"), HERE]
    from datetime import timedelta

    from dsv4attn.dist import SeqShard, SeqSplitPath, TorchDistComm
    from oracle_backend import OracleOps
    from seqsplit_case import load_shard, make_case, oracle_outputs

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        args, full, inputs = make_case(7, Bn, T_TOTAL, W, K, STEPS, POS0)
        shard = SeqShard(args, Bn, T_TOTAL, rank, world, "cpu", k=K, max_seq_len=MAX_SEQ, backend=OracleOps())
        load_shard(shard, full)
        shard.set_positions(POS0)
        path = SeqSplitPath(shard, TorchDistComm())
        want, _ = oracle_outputs(args, full, inputs, POS0, MAX_SEQ)
        for s, x in enumerate(inputs):
            if rank == fail_rank and s == 2:
                raise SystemExit(3)          # leaves between steps, nothing in flight
            out = torch.empty(Bn, args.n_heads, args.head_dim, dtype=torch.bfloat16)
            path.step([x], [out])
            err = (out.float() - want[s].float()).abs().max().item()
            assert torch.allclose(out.float(), want[s].float(), rtol=2e-2, atol=2e-2), (rank, s, err)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,Bn", [(2, 1), (3, 2)])
def test_seq_split_matches_unsplit_oracle(world, Bn):
    mp.spawn(_worker, args=(world, _free_port(), Bn, -1), nprocs=world, join=True)


def _exit_worker(rank, world, port, result_dir, leave_rank, leave_step):
    """One rank of a split in which rank ``leave_rank`` leaves between steps
    (nothing in flight); every other rank records how its own run ended in
    ``result_dir/rank<r>``: "ok", or "error <type>: <message>"."""
    sys.path[:0] = [os.path.dirname(HERE), os.path.join(os.path.dirname(HERE), "tt-deepseek-v4_b200"), HERE]
    import time
    from datetime import timedelta

    from dsv4attn.dist import SeqShard, SeqSplitPath, TorchDistComm
    from oracle_backend import OracleOps
    from seqsplit_case import load_shard, make_case

    # the rendezvous store lives in the test process, so the rank that
    # leaves (rank 0 included) takes no store down with it
    store = dist.TCPStore("127.0.0.1", port, is_master=False, timeout=timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=timedelta(seconds=5))
    res = "ok"
    t0 = time.time()
    try:
        args, full, inputs = make_case(7, 1, T_TOTAL, W, K, STEPS, POS0)
        shard = SeqShard(args, 1, T_TOTAL, rank, world, "cpu", k=K, max_seq_len=MAX_SEQ, backend=OracleOps())
        load_shard(shard, full)
        shard.set_positions(POS0)
        path = SeqSplitPath(shard, TorchDistComm())
        for s, x in enumerate(inputs):
            if rank == leave_rank and s == leave_step:
                raise SystemExit(3)
            out = torch.empty(1, args.n_heads, args.head_dim, dtype=torch.bfloat16)
            path.step([x], [out])
    except Exception as e:  # noqa: BLE001 - the failure itself is the result
        res = f"error {type(e).__name__}: {e}"
    finally:
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write(f"{time.time() - t0:.3f} {res}")
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


@pytest.mark.parametrize("world,leave_rank", [(2, 1), (3, 0)])
def test_seq_split_rank_exit_fails_the_others(tmp_path, world, leave_rank):
    """A rank that leaves between steps must make every surviving rank's own
    next exchange raise (within the process-group timeout), not hang and not
    return a wrong result."""
    ctx = mp.get_context("spawn")
    from datetime import timedelta
    store = dist.TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False, timeout=timedelta(seconds=60))
    port = store.port
    procs = [ctx.Process(target=_exit_worker, args=(r, world, port, str(tmp_path), leave_rank, 2))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=120)
        assert all(not p.is_alive() for p in procs), "a surviving rank hung"
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    assert procs[leave_rank].exitcode == 3
    for r in range(world):
        if r == leave_rank:
            continue
        text = (tmp_path / f"rank{r}").read_text()
        elapsed, res = text.split(" ", 1)
        assert res.startswith("error"), f"rank {r} did not fail: {res}"
        assert float(elapsed) < 60.0


def test_seq_shard_bounds_cover_the_context():
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "tt-deepseek-v4_b200"))
    from dsv4attn.dist import batch_shard, seq_shard
    for T in (1, 7, 96, 65536):
        for G in (1, 2, 3, 8):
            spans = [seq_shard(T, r, G) for r in range(G)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert batch_shard(64, 3, 8) == (24, 32)
    with pytest.raises(ValueError):
        batch_shard(64, 0, 3)
