"""Host-side logic of the row-sharded path on CPU: tile-aligned row ranges,
scale-slab placement, and the MAX all-reduce over a world-size-2 gloo group.
The per-shard quantization here is the oracle (the checker); the GPU path is
covered by the gpu-marked tests."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from test_speed_scalesweep_b200 import sharded


@pytest.mark.parametrize("total,world", [(524288, 8), (1000, 3), (129, 2), (128, 4), (5, 2)])
def test_shard_rows_cover_in_tiles(total, world):
    spans = [sharded.shard_rows(total, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == total
    for (a, b), (c, d) in zip(spans, spans[1:]):
        assert b == c
    for a, b in spans[:-1]:
        assert a % 128 == 0 and (b - a) % 128 == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, total, k, result_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests", "golden"))
    import golden_inputs as gi
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    full = gi.outlier_activations(total, k, seed=31)
    a, b = sharded.shard_rows(total, world, rank)
    mine = full[a:b]
    amax = torch.tensor([oracle.absmax(mine) if b > a else 0.0], dtype=torch.float32)
    sharded.all_reduce_amax(amax)
    gsi = oracle.global_scale_inv(float(amax.item()), 448.0)
    codes, scales = oracle.quantize(mine, gsi)
    np.savez(os.path.join(result_dir, f"r{rank}.npz"), codes=codes, scales=scales,
             span=np.array([a, b]), gsi=np.array([gsi], np.float32))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("total,world", [(300, 2), (256, 2)])
def test_two_rank_gloo_shards_reassemble_to_whole_tensor(tmp_path, total, world):
    import golden_inputs as gi
    import oracle
    k = 256
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, total, k, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    full = gi.outlier_activations(total, k, seed=31)
    gsi = oracle.global_scale_inv(oracle.absmax(full), 448.0)
    whole_codes, whole_scales = oracle.quantize(full, gsi)
    codes, slabs = [], []
    for r in range(world):
        d = np.load(tmp_path / f"r{r}.npz")
        assert np.float32(d["gsi"][0]) == np.float32(gsi)
        codes.append(d["codes"])
        a, b = d["span"]
        lo, hi = sharded.scale_slab_rows(int(a), int(b))
        kpad = whole_scales.shape[1]
        assert d["scales"].shape == (hi - lo, kpad)
        slabs.append(d["scales"])
    assert np.array_equal(np.concatenate(codes), whole_codes)
    assert np.array_equal(np.concatenate(slabs), whole_scales)


def _dying_worker(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves between steps, before the collective
    amax = torch.ones(1)
    try:
        sharded.all_reduce_amax(amax)
    except Exception:
        os._exit(17)  # the surviving rank sees an error instead of hanging
    os._exit(0)


def test_missing_rank_surfaces_as_an_error_not_a_hang():
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert procs[0].exitcode == 17


def _amax_worker(rank, world, port, values, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    amax = torch.tensor([values[rank]], dtype=torch.float32)
    sharded.all_reduce_amax(amax)
    np.save(os.path.join(result_dir, f"a{rank}.npy"), amax.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("values,want", [
    ((3.5, float("nan")), "nan"),          # NaN on the second rank
    ((float("nan"), 1e30), "nan"),         # NaN on the first rank
    ((float("inf"), 2.0), float("inf")),
    ((0.0, 0.0), 0.0),
    ((7.25, 1e-40), 7.25),                 # a subnormal amax loses to a normal one
])
def test_amax_all_reduce_carries_nan_and_inf(tmp_path, values, want):
    """A NaN in any shard must make the tensor-wide amax NaN on every rank,
    as x.abs().max() over the whole tensor does (the gsi then follows it)."""
    port = _free_port()
    mp.start_processes(_amax_worker, args=(2, port, values, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    for r in range(2):
        got = float(np.load(tmp_path / f"a{r}.npy")[0])
        if want == "nan":
            assert np.isnan(got), got
        else:
            assert got == want, got


def test_amax_all_reduce_rejects_non_float32():
    with pytest.raises(ValueError):
        sharded.all_reduce_amax(torch.zeros(1, dtype=torch.float64))
