"""The (batch, head) split of one attention call across ranks (mlx_primitives.attention.partition)
on CPU ranks over gloo (127.0.0.1): world sizes 2, 3 and 4, both layouts, grouped K/V heads,
a broadcast K/V batch, unit counts that do not divide evenly.  Each rank runs only its own
units, with the CPU oracle standing in for the kernel launch; the test checks that every
(batch, head) unit is computed by exactly one rank and that the reassembled output equals the
oracle's whole-call attention."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention_oracle as O


def oracle_backend(q, k, v, *, layout, scale, causal, window_left, window_right, q_offset,
                   kv_offset, kv_splits, out):
    """attention_forward's arguments plus ``out``: the oracle in fp64, written in place."""
    qb, kb, vb = (O.to_bhsd(t.double().numpy(), layout) for t in (q, k, v))
    group = qb.shape[1] // kb.shape[1]
    kb, vb = (np.repeat(t, group, axis=1) for t in (kb, vb))
    if kb.shape[0] != qb.shape[0]:
        kb, vb = (np.broadcast_to(t, (qb.shape[0],) + t.shape[1:]) for t in (kb, vb))
    o = O.attention_bhsd(qb, kb, vb, scale, causal=causal, window_left=window_left,
                         window_right=window_right, q_offset=q_offset, kv_offset=kv_offset)
    out.copy_(torch.from_numpy(np.ascontiguousarray(O.from_bhsd(o, layout))))


CASES = {
    # name: (layout, B, H, H_kv, Sq, Skv, D, kind)
    "flash_bhsd": ("BHSD", 3, 5, 5, 40, 40, 16, "flash"),
    "flash_bshd_gqa": ("BSHD", 2, 6, 2, 24, 36, 16, "flash"),
    "window_bshd": ("BSHD", 2, 4, 4, 48, 48, 8, "window"),
    "chunked_bshd_bcast_kv": ("BSHD", 3, 4, 4, 12, 64, 8, "chunked"),
}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, errq):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from mlx_primitives.attention.partition import attention_units, shard_units

        layout, B, H, Hkv, Sq, Skv, D, kind = CASES[case]
        Bk = 1 if "bcast" in case else B
        shp = lambda b, h, s: (b, h, s, D) if layout == "BHSD" else (b, s, h, D)
        q = torch.from_numpy(O.make_qkv(shp(B, H, Sq), (1, 1, 1, 1), seed=3)[0])
        k, v = (torch.from_numpy(a) for a in O.make_qkv(shp(Bk, Hkv, Skv), shp(Bk, Hkv, Skv),
                                                        seed=4)[1:])
        mask = {"flash": dict(causal=True, q_offset=Skv - Sq),
                "window": dict(causal=True, window_left=5),
                "chunked": dict(causal=False)}[kind]
        scale = D ** -0.5

        units = shard_units(B, H, world, rank)
        out = torch.zeros(q.shape, dtype=torch.float32)
        attention_units(q, k, v, units, layout=layout, scale=scale, out=out,
                        backend=oracle_backend, **mask)
        # unit coverage: each rank marks the units it computed
        cover = torch.zeros(B * H, dtype=torch.int64)
        cover[units.start:units.stop] += 1
        dist.all_reduce(cover)
        if not torch.equal(cover, torch.ones_like(cover)):
            raise AssertionError(f"unit coverage {cover.tolist()}")
        # the rows a rank did not compute stay zero, so the sum over ranks is the whole output
        dist.all_reduce(out)
        want = torch.zeros_like(out)
        full = dict(dict(window_left=-1, window_right=-1, q_offset=0, kv_offset=0), **mask)
        oracle_backend(q, k, v, layout=layout, scale=scale, kv_splits=0, out=want, **full)
        err = (out - want).abs().max().item()
        if err > 1e-6:
            raise AssertionError(f"rank {rank}: max-abs {err}")
        dist.barrier()
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001 - reported to the parent
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")


@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("case", sorted(CASES))
def test_units_split_covers_every_unit_once(world, case):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, errq)) for r in range(world)]
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


@pytest.mark.parametrize("B,H,world", [(4, 32, 8), (2, 32, 8), (8, 16, 8), (2, 12, 8),
                                       (3, 5, 4), (1, 7, 3), (1, 1, 2)])
def test_shard_units_is_a_balanced_partition(B, H, world):
    from mlx_primitives.attention.partition import shard_units, unit_blocks

    seen, sizes = [], []
    for r in range(world):
        units = shard_units(B, H, world, r)
        sizes.append(len(units))
        blocks = unit_blocks(units, H)
        assert len(blocks) <= 3
        for b0, b1, h0, h1 in blocks:
            seen += [b * H + h for b in range(b0, b1) for h in range(h0, h1)]
    assert sorted(seen) == list(range(B * H))
    assert max(sizes) - min(sizes) <= 1


def test_group_pieces_split_at_kv_group_boundaries():
    from mlx_primitives.attention.partition import _group_pieces

    assert _group_pieces(3, 13, 4) == [(3, 4), (4, 12), (12, 13)]
    assert _group_pieces(0, 2, 3) == [(0, 2)]
    assert _group_pieces(4, 6, 3) == [(4, 6)]
    assert _group_pieces(2, 6, 4) == [(2, 4), (4, 6)]
    assert _group_pieces(0, 32, 1) == [(0, 32)]


def test_baseline_shapes_take_one_launch_per_rank():
    """Configs 2, 3 and 4 at 1, 2, 4 and 8 ranks: one rectangle, i.e. one kernel launch."""
    from mlx_primitives.attention.partition import shard_units, unit_blocks

    for B, H in ((4, 32), (2, 32), (8, 16)):
        for world in (1, 2, 4, 8):
            for r in range(world):
                assert len(unit_blocks(shard_units(B, H, world, r), H)) == 1
