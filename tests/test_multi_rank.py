"""Multi-process (gloo, CPU, world size 2) tests of the N-sharding and output
gather logic, and of failure detection on the host: a rank that fails before
the collective makes the other rank's collective end with an error instead
of hanging."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wide_compiler import parallel


def test_shard_range_partitions():
    for n in (1, 5, 64, 100):
        for world in (1, 2, 3, 8):
            spans = [parallel.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    assert [b - a for a, b in (parallel.shard_range(100, 8, r) for r in range(8))] == [13] * 4 + [12] * 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n_total, fail_rank, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    try:
        full = torch.arange(n_total * 3 * 2, dtype=torch.float32).view(n_total, 3, 2)
        a, b = parallel.shard_range(n_total, world, rank)
        models = list(range(n_total))
        assert parallel.shard_models(models) == models[a:b]
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        got = parallel.gather_outputs(full[a:b] * 1.0, n_total)
        # channel-packed outputs [B, n_local*F, S] -> [B, N*F, S]
        bsz, f, sp = 3, 2, 5
        packed_full = torch.arange(bsz * n_total * f * sp, dtype=torch.float32).view(bsz, n_total * f, sp)
        got_p = parallel.gather_packed(packed_full[:, a * f:b * f].contiguous(), n_total)
        # the overlapped form ShardedWideModel(gather_chunks=2) uses: two batch
        # slices gathered asynchronously, then placed into slices of the result
        chunked = torch.empty_like(packed_full)
        places = []
        for c in range(2):
            b0, b1 = parallel.shard_range(bsz, 2, c)
            places.append((b0, b1, parallel._start_gather_packed(packed_full[b0:b1, a * f:b * f].contiguous(),
                                                                  n_total)))
        for b0, b1, place in places:
            place(chunked[b0:b1])
        ok = bool(torch.equal(got, full)) and bool(torch.equal(got_p, packed_full)) and \
            bool(torch.equal(chunked, packed_full))
        torch.save({"ok": ok}, f"{result_path}.{rank}")
    except Exception as e:  # report on the host, never on a device
        torch.save({"ok": False, "error": repr(e)}, f"{result_path}.{rank}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, n_total, fail_rank, tmp_path):
    path = str(tmp_path / "res")
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, n_total, fail_rank, path)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    return [torch.load(f"{path}.{r}") for r in range(world)]


@pytest.mark.parametrize("n_total", [4, 5])
def test_gather_outputs_gloo_world2(tmp_path, n_total):
    """Even (4) and ragged (5) splits of N-first and channel-packed outputs."""
    res = _run(2, n_total, -1, tmp_path)
    assert all(r["ok"] for r in res), res


def test_failed_rank_is_detected_not_hung(tmp_path):
    res = _run(2, 6, 1, tmp_path)
    assert not res[1]["ok"] and "injected" in res[1]["error"]
    assert not res[0]["ok"] and "error" in res[0]      # rank 0's collective errored (timeout / peer closed)


def test_copy_rows_slices_a_rank_s_channels():
    """The strided copy that cuts one rank's channel range out of the full
    packed input (the CPU form of the device kernel's addressing)."""
    n_total, c, bsz, sp = 7, 3, 4, 6
    x = torch.randn(bsz, n_total * c, sp)
    for world in (2, 3):
        for rank in range(world):
            lo, hi = parallel.shard_range(n_total, world, rank)
            inner = c * sp
            out = torch.empty(bsz, (hi - lo) * c, sp)
            parallel.copy_rows(x.view(bsz, -1)[:, lo * inner:], n_total * inner * 4, out, (hi - lo) * inner * 4,
                               bsz, (hi - lo) * inner * 4)
            assert torch.equal(out, x[:, lo * c:hi * c])
