"""Multi-GPU tests (skipped with fewer than 2 GPUs): the sequence-parallel ring over NCCL
against single-GPU flash attention of the full sequence, per rank, bf16 tolerance 2e-2."""

import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ring_worker(rank, world, port, shape, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        from datetime import timedelta
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        import mlx_primitives as mp_
        from mlx_primitives.attention.ring import ring_flash_attention, zigzag_shard

        B, H, S, D = shape
        g = torch.Generator(device=dev)
        g.manual_seed(77)
        q, k, v = (torch.randn(shape, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
        want = mp_.flash_attention(q, k, v, causal=True, layout="BHSD")
        shard = lambda t: zigzag_shard(t, world, rank).contiguous()
        out = ring_flash_attention(shard(q), shard(k), shard(v))
        torch.cuda.synchronize()
        err = (out.float() - shard(want).float()).abs().max().item()
        if not err <= 2e-2:
            raise AssertionError(f"rank {rank}: max-abs {err}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("S", [8192, 8192 + 2 * 2 * 256])
def test_ring_two_gpus_matches_single_gpu(S):
    world = 2
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ring_worker, args=(r, world, port, (1, 4, S, 128), errq))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
