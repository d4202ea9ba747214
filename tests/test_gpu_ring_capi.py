"""The C-ABI ring (mlxp_ring_*: NCCL loaded by the library, no torch.distributed) against
single-GPU flash attention of the whole sequence and, for two ranks, against the fp64 oracle on
every zig-zag chunk boundary, bf16 tolerance 2e-2.  One rank runs on one
GPU (a ring of one is plain causal attention of the shard, which is then the whole sequence);
two ranks need two GPUs and are skipped otherwise."""

import os
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _inputs(shape, dev, seed=5):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return [torch.randn(shape, generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]


@pytest.mark.parametrize("layout", ["BHSD", "BSHD"])
def test_ring_capi_single_rank_is_causal_attention(layout):
    import mlx_primitives as mp_
    from mlx_primitives.attention.ring import NcclRing, nccl_unique_id

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    B, H, S, D = 2, 4, 1024, 128
    q, k, v = _inputs((B, H, S, D), dev)
    if layout == "BSHD":
        q, k, v = (t.transpose(1, 2).contiguous() for t in (q, k, v))
    want = mp_.flash_attention(q, k, v, causal=True, layout=layout)
    with NcclRing(nccl_unique_id(), 1, 0) as ring:
        got = ring.forward(q, k, v, layout=layout)
        again = ring.forward(q, k, v, layout=layout)
    torch.cuda.synchronize()
    assert (got.float() - want.float()).abs().max().item() <= 2e-2
    assert torch.equal(got, again)


def test_ring_capi_rejects_bad_shapes():
    from mlx_primitives.attention.ring import NcclRing, nccl_unique_id

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    q, k, v = _inputs((1, 2, 7, 64), dev)  # odd local length: not two equal chunks
    with NcclRing(nccl_unique_id(), 1, 0) as ring:
        with pytest.raises(ValueError):
            ring.forward(q, k, v)


def _worker(rank, world, uid, shape, errq):
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        import mlx_primitives as mp_
        from mlx_primitives.attention.ring import NcclRing, zigzag_shard

        from test_gpu_multi import check_shard_vs_oracle

        q, k, v = _inputs(shape, dev, seed=9)
        want = zigzag_shard(mp_.flash_attention(q, k, v, causal=True, layout="BHSD"), world,
                            rank)
        shard = lambda t: zigzag_shard(t, world, rank).contiguous()
        with NcclRing(uid, world, rank) as ring:
            out = ring.forward(shard(q), shard(k), shard(v))
            torch.cuda.synchronize()
        # the fp64 oracle on every zig-zag chunk boundary of this rank's chunks, all heads
        check_shard_vs_oracle(out, q, k, v, range(shape[1]), shape[2], world, rank,
                              shape[3] ** -0.5)
        err = (out.float() - want.float()).abs().max().item()
        if not err <= 2e-2:
            raise AssertionError(f"rank {rank}: max-abs {err}")
    except Exception:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ring_capi_two_ranks_match_single_gpu():
    from mlx_primitives.attention.ring import nccl_unique_id

    world = 2
    uid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, uid, (1, 4, 8192, 128), errq))
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
