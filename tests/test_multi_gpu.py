"""Row-sharded quantization on 2+ GPUs over NCCL: the concatenated shards must
equal the single-GPU quantization of the whole tensor, byte for byte.  Skips
unless the machine has at least two GPUs."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

ROWS, K = 1000, 4096  # 1000 rows: the last rank's shard is not a multiple of 128


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _make_input(device):
    g = torch.Generator(device=device).manual_seed(2024)
    x = torch.randn(ROWS, K, generator=g, device=device).to(torch.bfloat16)
    x[:, ::200] *= 20
    x[777, 5] = 3000.0  # the global max lives in the last shard
    return x


def _rank(rank, world, port, out_dir, backend_name):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from datetime import timedelta

    import torch.distributed as dist

    from test_speed_scalesweep_b200 import sharded
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    x = _make_input(dev)
    a, b = sharded.shard_rows(ROWS, world, rank)
    codes, scales, gsi = sharded.quantize_row_shard(x[a:b].contiguous(), 448.0,
                                                    backend=backend_name)
    torch.cuda.synchronize()
    torch.save({"codes": codes.cpu(), "scales": scales.view(torch.uint8).cpu(), "gsi": gsi.cpu(),
                "span": (a, b)}, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("backend_name", ["scalesweep_mse", "scalesweep_mse_reference"])
def test_row_sharded_equals_single_gpu(tmp_path, backend_name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs at least two GPUs")
    import torch.multiprocessing as mp

    from test_speed_scalesweep_b200 import custom, global_scale
    world = min(torch.cuda.device_count(), 4)
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path), backend_name),
                       nprocs=world, start_method="spawn", join=True)
    x = _make_input(torch.device("cuda", 0))
    gsi = global_scale.global_scale_inv_from_max(x, 448.0)
    codes, scales = custom.nvfp4_quant(x, gsi, True, backend_name)
    parts = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    for p in parts:
        assert p["gsi"].view(torch.int32).item() == gsi.cpu().view(torch.int32).item()
    assert torch.equal(torch.cat([p["codes"] for p in parts]), codes.cpu())
    # each rank's swizzled slab is the matching slice of the whole buffer; only
    # the bytes a shard writes (its valid rows) are defined
    import numpy as np

    import golden_inputs as gi
    whole = scales.view(torch.uint8).cpu().numpy()
    for p in parts:
        a, b = p["span"]
        slab = p["scales"].numpy()
        assert a % 128 == 0 and slab.shape[1] == whole.shape[1]
        mask = gi.written_scale_mask(dict(m=b - a, k=K), "mse", True, slab.shape)
        assert np.array_equal(slab[mask], whole[a: a + slab.shape[0]][mask])
