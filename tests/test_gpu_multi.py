"""Multi-GPU tests (skipped when the box has fewer GPUs than ranks), one process per GPU over
NCCL (NVLS off), bf16 tolerance 2e-2 max-abs.

Ring (sequence-parallel zig-zag, mlx_primitives.attention.ring): each rank's output shard is
checked (a) against the exact fp64 oracle on sampled rows — row 0, row S-1, the first and last
row of every one of the 2P zig-zag chunks and random rows, each rank checking the rows of the
two chunks it holds, on sampled heads — and (b) against single-GPU flash attention of the whole
sequence.  Shapes: S = 8192 and a ragged 9216 at P = 2, and BASELINE config 5 itself (one
131072-token sequence, 32 heads, head_dim 128) at P = 2, 4 and 8.

(Batch, head) split (mlx_primitives.attention.partition): every rank computes only its own
units of config 2's shape; the outputs summed over ranks (a test-only all-reduce: the split
itself has no collective) must equal the single-GPU call bit for bit, and each rank's units
must match the oracle on sampled rows."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=timedelta(seconds=120), device_id=dev)
    return dev


def zigzag_check_rows(S, world, n_random=6, seed=0):
    """Global rows to check: 0, S-1, the first two and the last row of each of the 2P chunks,
    and random rows."""
    C = S // (2 * world)
    rows = {0, S - 1}
    for c in range(2 * world):
        rows |= {c * C, c * C + 1, (c + 1) * C - 1}
    rows |= set(np.random.RandomState(seed).randint(0, S, n_random).tolist())
    return np.array(sorted(rows))


def local_rows(rows, S, world, rank):
    """(global rows, local indices) of the rows that `rank` holds in its zig-zag shard."""
    C = S // (2 * world)
    a, b = rank, 2 * world - 1 - rank
    g, loc = [], []
    for r in rows:
        c = r // C
        if c == a:
            g.append(r)
            loc.append(r - a * C)
        elif c == b:
            g.append(r)
            loc.append(C + r - b * C)
    return np.array(g, dtype=np.int64), np.array(loc, dtype=np.int64)


def check_shard_vs_oracle(out_shard, q, k, v, heads, S, world, rank, scale):
    """out_shard: this rank's BHSD shard; q, k, v: the whole sequence (BHSD, B = 1)."""
    from oracle import attention_oracle as O

    rows, loc = local_rows(zigzag_check_rows(S, world), S, world, rank)
    for h in heads:
        want = O.attention_rows_bhsd(q[:1, h:h + 1].float().cpu().numpy(),
                                     k[:1, h:h + 1].float().cpu().numpy(),
                                     v[:1, h:h + 1].float().cpu().numpy(), rows, scale,
                                     causal=True)[0]
        got = out_shard[0, h, torch.as_tensor(loc, device=out_shard.device)].float().cpu().numpy()
        err = np.abs(got - want).max()
        if not err <= TOL:
            raise AssertionError(f"rank {rank} head {h}: max-abs {err} vs the fp64 oracle")


def _ring_worker(rank, world, port, shape, heads, errq):
    try:
        dev = _init(rank, world, port)
        import mlx_primitives as mp_
        from mlx_primitives.attention.ring import ring_flash_attention, zigzag_shard

        B, H, S, D = shape
        g = torch.Generator(device=dev)
        g.manual_seed(77)
        q, k, v = (torch.randn(shape, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
        shard = lambda t: zigzag_shard(t, world, rank).contiguous()
        out = ring_flash_attention(shard(q), shard(k), shard(v))
        torch.cuda.synchronize()
        check_shard_vs_oracle(out, q, k, v, heads, S, world, rank, D ** -0.5)
        want = mp_.flash_attention(q, k, v, causal=True, layout="BHSD")
        err = (out.float() - shard(want).float()).abs().max().item()
        if not err <= TOL:
            raise AssertionError(f"rank {rank}: max-abs {err} vs single-GPU attention")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")


def _run(target, world, args, timeout=600):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("S", [8192, 8192 + 2 * 2 * 256])
def test_ring_two_gpus_matches_oracle_and_single_gpu(S):
    _run(_ring_worker, 2, ((1, 4, S, 128), (0, 1, 2, 3)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ring_config5_128k_matches_oracle(world):
    """one 131072-token sequence, 32 heads, head_dim 128, as a P-rank ring."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run(_ring_worker, world, ((1, 32, 131072, 128), (0, 13, 31)), timeout=900)


def _partition_worker(rank, world, port, errq):
    try:
        dev = _init(rank, world, port)
        import mlx_primitives as mp_
        from mlx_primitives.attention import flash_attention_shard, shard_units
        from oracle import attention_oracle as O

        B, H, S, D = 4, 32, 4096, 128  # config 2's shape
        g = torch.Generator(device=dev)
        g.manual_seed(42)
        q, k, v = (torch.randn((B, H, S, D), generator=g, device=dev).to(torch.bfloat16)
                   for _ in range(3))
        out = torch.zeros_like(q)
        flash_attention_shard(q, k, v, world, rank, causal=True, layout="BHSD", out=out)
        torch.cuda.synchronize()
        units = shard_units(B, H, world, rank)
        rows = np.array([0, 1, 127, 128, 255, 256, 2047, 2048, S - 129, S - 128, S - 1])
        for u in (units.start, (units.start + units.stop) // 2, units.stop - 1):
            b, h = divmod(u, H)
            want = O.attention_rows_bhsd(q[b:b + 1, h:h + 1].float().cpu().numpy(),
                                         k[b:b + 1, h:h + 1].float().cpu().numpy(),
                                         v[b:b + 1, h:h + 1].float().cpu().numpy(), rows,
                                         D ** -0.5, causal=True)[0]
            got = out[b, h, torch.as_tensor(rows, device=dev)].float().cpu().numpy()
            err = np.abs(got - want).max()
            if not err <= TOL:
                raise AssertionError(f"rank {rank} unit {u}: max-abs {err} vs the fp64 oracle")
        dist.all_reduce(out)  # test only: reassemble (every other rank's rows are zero)
        whole = mp_.flash_attention(q, k, v, causal=True, layout="BHSD")
        if not torch.equal(out, whole):
            raise AssertionError(f"rank {rank}: reassembled split differs from the whole call")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_batch_head_split_of_config2(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run(_partition_worker, world, ())
