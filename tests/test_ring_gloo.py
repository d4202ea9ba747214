"""Multi-rank tests of the sequence-parallel ring (mlx_primitives.attention.ring) on CPU ranks:
world_size 2 and 3 over gloo on 127.0.0.1, the real ring driver (zig-zag schedule, P2P
send/recv of K/V blocks, double buffering, LSE merging) with the CPU oracle as the compute
backend.  Each rank's output shard must equal the oracle's full causal attention restricted
to that rank's chunks."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention_oracle as O


class OracleRingBackend:
    """Partial attention / merge / cast on the CPU with the oracle (fp64), in place."""

    def partial(self, q, k, v, scale, q_off, kv_off, o_part, lse_part):
        o, lse = O.attention_bhsd(q.double().numpy(), k.double().numpy(), v.double().numpy(),
                                  scale, causal=True, q_offset=q_off, kv_offset=kv_off,
                                  return_lse=True)
        o_part.copy_(torch.from_numpy(o))
        lse_part.copy_(torch.from_numpy(lse))

    def merge(self, o_acc, lse_acc, o_new, lse_new):
        o, lse = O.lse_merge(np.stack([o_acc.numpy(), o_new.numpy()]),
                             np.stack([lse_acc.numpy(), lse_new.numpy()]))
        o_acc.copy_(torch.from_numpy(o))
        lse_acc.copy_(torch.from_numpy(lse))

    def finish(self, o_acc, out):
        out.copy_(o_acc)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, shape, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from mlx_primitives.attention.ring import ring_flash_attention, zigzag_shard

        B, H, S, D = shape
        q, k, v = (torch.from_numpy(a) for a in O.make_qkv((B, H, S, D), (B, H, S, D), seed=31))
        scale = 0.17
        want = torch.from_numpy(O.attention_bhsd(q.numpy(), k.numpy(), v.numpy(), scale,
                                                 causal=True)).float()
        shard = lambda t: zigzag_shard(t, world, rank).contiguous()
        out = ring_flash_attention(shard(q), shard(k), shard(v), scale=scale,
                                   backend=OracleRingBackend())
        err = (out - shard(want)).abs().max().item()
        if err > 1e-5:
            raise AssertionError(f"rank {rank}: max-abs {err}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")


@pytest.mark.parametrize("world", [2, 3])
def test_ring_matches_full_causal_attention_on_cpu_ranks(world):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    S = 16 * 2 * world
    procs = [ctx.Process(target=_worker, args=(r, world, port, (1, 2, S, 32), errq))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_zigzag_shard_roundtrip():
    from mlx_primitives.attention.ring import zigzag_shard, zigzag_unshard

    x = torch.arange(2 * 3 * 24 * 4).reshape(2, 3, 24, 4)
    parts = [zigzag_shard(x, 3, r) for r in range(3)]
    assert torch.equal(zigzag_unshard(parts), x)
    assert torch.equal(parts[0][:, :, :4], x[:, :, 0:4]) and torch.equal(parts[0][:, :, 4:], x[:, :, 20:24])
