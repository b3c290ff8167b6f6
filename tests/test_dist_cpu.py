"""CPU (gloo, world size 2 to 8) checks of the multi-GPU row sharding.

The block shards video tokens by rows; every per-row op stays local and the
K/V rows that attention reads from all ranks are all-gathered
(``RowShard.gather_rows``).  These tests run the same composition as
``QAttention.core`` on CPU ranks -- RoPE on the local rows, gather of the
rotated K and of V, attention of the local queries -- and check that the
concatenated per-rank outputs equal the unsharded computation, and that a
rank that never joins makes the others fail with a timeout instead of
hanging.
"""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rope(x, pe, heads):
    from ltxq.block import apply_split_rope

    return apply_split_rope(x, pe, heads)


def _attention(q, k, v, heads):
    b, tq, w = q.shape
    d = w // heads
    qh = q.float().view(b, tq, heads, d).transpose(1, 2)
    kh = k.float().view(b, k.shape[1], heads, d).transpose(1, 2)
    vh = v.float().view(b, v.shape[1], heads, d).transpose(1, 2)
    o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)
    return o.transpose(1, 2).reshape(b, tq, w)


def _case(T=48, heads=4, d=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    w = heads * d
    q = torch.randn(1, T, w, generator=g).to(torch.bfloat16)
    k = torch.randn(1, T, w, generator=g).to(torch.bfloat16)
    v = torch.randn(1, T, w, generator=g).to(torch.bfloat16)
    ang = torch.rand(1, heads, T, d // 2, generator=g) * 6.28
    return q, k, v, (torch.cos(ang), torch.sin(ang)), heads


def _worker(rank, world, port, out_dir):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ltx-2-mlx_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from ltxq.block import RowShard

    q, k, v, pe, heads = _case()
    T = q.shape[1]
    tl = T // world
    rows = slice(rank * tl, (rank + 1) * tl)
    pe_l = tuple(c[:, :, rows].contiguous() for c in pe)
    shard = RowShard(dist.group.WORLD, world, rank)
    ql = _rope(q[:, rows], pe_l, heads)
    kl = _rope(k[:, rows], pe_l, heads)
    kg = shard.gather_rows(kl)
    vg = shard.gather_rows(v[:, rows].contiguous())
    o = _attention(ql, kg, vg, heads)
    torch.save({"o": o, "kg": kg}, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_row_sharded_attention_equals_unsharded(tmp_path, world):
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    q, k, v, pe, heads = _case()
    ref_k = _rope(k, pe, heads)
    ref = _attention(_rope(q, pe, heads), ref_k, v, heads)
    outs = [torch.load(os.path.join(tmp_path, f"rank{r}.pt")) for r in range(world)]
    got = torch.cat([o["o"] for o in outs], dim=1)
    assert torch.equal(outs[0]["kg"], ref_k)  # every rank sees the full rotated K
    assert torch.allclose(got, ref, atol=1e-5, rtol=1e-5)


def _batch_worker(rank, world, port, out_dir):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ltx-2-mlx_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from ltxq.block import RowShard

    g = torch.Generator().manual_seed(7)
    full_k = torch.randn(2, 8 * world, 6, generator=g)
    full_v = torch.randn(2, 8 * world, 6, generator=g)
    rows = slice(rank * 8, (rank + 1) * 8)
    shard = RowShard(dist.group.WORLD, world, rank)
    k, v = shard.finish_gather(shard.start_gather(full_k[:, rows], full_v[:, rows], overlap=False))
    torch.save({"k": k, "v": v, "full_k": full_k, "full_v": full_v}, os.path.join(out_dir, f"b{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_batched_gather_restores_row_order(tmp_path):
    """Batch 2: every rank's gathered K/V equal the unsharded tensors (the
    rank-major blocks are put back in row order per batch entry)."""
    world = 2
    port = _free_port()
    mp.start_processes(_batch_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(world):
        o = torch.load(os.path.join(tmp_path, f"b{r}.pt"))
        assert torch.equal(o["k"], o["full_k"]) and torch.equal(o["v"], o["full_v"])


def _lonely_worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    if rank == 1:
        return  # this rank never joins
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
        open(os.path.join(out_dir, "joined"), "w").close()
    except Exception as e:  # the rendezvous times out instead of hanging
        with open(os.path.join(out_dir, "error"), "w") as f:
            f.write(type(e).__name__)


def test_missing_rank_times_out_on_host(tmp_path):
    port = _free_port()
    mp.start_processes(_lonely_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert os.path.exists(os.path.join(tmp_path, "error"))
    assert not os.path.exists(os.path.join(tmp_path, "joined"))


def _hp_worker(rank, world, port, out_dir):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ltx-2-mlx_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from ltxq.block import (RowShard, heads_to_ranks, merge_attention_partials, ranks_to_heads,
                            ranks_to_sequence, sequence_to_ranks)

    q, k, v, _, heads = _case()
    q, k, v = q.float(), k.float(), v.float()
    T = q.shape[1]
    tl = T // world
    rows = slice(rank * tl, (rank + 1) * tl)
    shard = RowShard(dist.group.WORLD, world, rank, overlap=False)
    calls = []
    shard.wait_probe = lambda kind, phase: calls.append((kind, phase))
    # head-parallel self-attention: Q/K/V rows -> heads, attention, back to rows
    send = torch.stack([heads_to_ranks(t[:, rows].contiguous(), world, heads) for t in (q, k, v)], dim=1)
    recv = shard.all_to_all(send)
    qh, kh, vh = (ranks_to_sequence(recv[:, i]) for i in range(3))
    o = torch.nn.functional.scaled_dot_product_attention(qh, kh, vh)
    hp = ranks_to_heads(shard.all_to_all(sequence_to_ranks(o, world)))
    # replicated queries over row-split keys, merged by log-sum-exp
    d = q.shape[2] // heads
    qf = q.view(1, T, heads, d).transpose(1, 2)
    kl = k[:, rows].reshape(1, tl, heads, d).transpose(1, 2)
    vl = v[:, rows].reshape(1, tl, heads, d).transpose(1, 2)
    sc = (qf @ kl.transpose(-1, -2)) / d ** 0.5
    lse = torch.logsumexp(sc, dim=-1)
    part_o = torch.softmax(sc, dim=-1) @ vl
    outs = torch.empty(world * part_o.numel())
    lses = torch.empty(world * lse.numel())
    dist.all_gather_into_tensor(outs, part_o.contiguous().flatten())
    dist.all_gather_into_tensor(lses, lse.contiguous().flatten())
    merged = merge_attention_partials(outs.view((world,) + tuple(part_o.shape)),
                                      lses.view((world,) + tuple(lse.shape)))
    kg = shard.gather_rows(k[:, rows].contiguous())  # in-line all-gather (overlap off)
    torch.save({"hp": hp, "merged": merged, "calls": calls, "kg": kg}, os.path.join(out_dir, f"hp{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_parallel_and_split_key_attention(tmp_path, world):
    """The two sharded attention forms of the block: head-parallel
    self-attention (all-to-all of Q/K/V rows to heads and back) equals the
    unsharded attention on each rank's rows; replicated queries over row-split
    keys, merged by log-sum-exp, equal attention over all keys.  The
    exchange probe (``RowShard.wait_probe``) is called around every in-line
    collective."""
    port = _free_port()
    mp.start_processes(_hp_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True, start_method="spawn")
    q, k, v, _, heads = _case()
    q, k, v = q.float(), k.float(), v.float()
    full = _attention(q, k, v, heads)
    T = q.shape[1]
    tl = T // world
    d = q.shape[2] // heads
    ref_merged = torch.nn.functional.scaled_dot_product_attention(
        q.view(1, T, heads, d).transpose(1, 2), k.view(1, T, heads, d).transpose(1, 2),
        v.view(1, T, heads, d).transpose(1, 2))
    for r in range(world):
        o = torch.load(os.path.join(tmp_path, f"hp{r}.pt"))
        assert torch.allclose(o["hp"], full[:, r * tl:(r + 1) * tl], atol=1e-5, rtol=1e-5)
        assert torch.allclose(o["merged"], ref_merged, atol=1e-5, rtol=1e-5)
        assert torch.equal(o["kg"], k)
        # the exchange probe brackets each in-line collective: two all-to-alls, one all-gather
        assert o["calls"] == [("sync", 0), ("sync", 1)] * 3


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_parallel_layouts_with_an_emulated_all_to_all(world):
    """heads_to_ranks -> all-to-all -> ranks_to_sequence gives each rank its
    H/world heads over all tokens in global order, and sequence_to_ranks ->
    all-to-all -> ranks_to_heads gives each rank back its token rows with all
    heads; the all-to-all is emulated in process (block g of rank r's send
    buffer becomes block r of rank g's receive buffer)."""
    from ltxq.block import heads_to_ranks, ranks_to_heads, ranks_to_sequence, sequence_to_ranks

    B, T, H, D = 2, 48, 8, 16
    g = torch.Generator().manual_seed(world)
    x = torch.randn(B, T, H * D, generator=g)
    tl = T // world
    sends = [heads_to_ranks(x[:, r * tl:(r + 1) * tl].contiguous(), world, H) for r in range(world)]
    recvs = [torch.stack([sends[src][dst] for src in range(world)]) for dst in range(world)]
    full = x.view(B, T, H, D).transpose(1, 2)  # (B, H, T, D)
    hw = H // world
    for r in range(world):
        seq = ranks_to_sequence(recvs[r])
        assert torch.equal(seq, full[:, r * hw:(r + 1) * hw])
    outs = [sequence_to_ranks(full[:, r * hw:(r + 1) * hw].contiguous(), world) for r in range(world)]
    backs = [torch.stack([outs[src][dst] for src in range(world)]) for dst in range(world)]
    for r in range(world):
        assert torch.equal(ranks_to_heads(backs[r]), x[:, r * tl:(r + 1) * tl])


@pytest.mark.parametrize("parts", [1, 3, 8])
def test_lse_merge_of_key_partitions(parts):
    """merge_attention_partials over any number of key partitions (uneven
    ones included) equals attention over all keys."""
    from ltxq.block import merge_attention_partials

    g = torch.Generator().manual_seed(parts)
    B, H, Lq, Lk, D = 1, 4, 20, 64, 16
    q, k, v = (torch.randn(B, H, n, D, generator=g) for n in (Lq, Lk, Lk))
    bounds = torch.linspace(0, Lk, parts + 1).round().long().tolist()
    outs, lses = [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        sc = (q @ k[:, :, a:b].transpose(-1, -2)) / D ** 0.5
        lses.append(torch.logsumexp(sc, dim=-1))
        outs.append(torch.softmax(sc, dim=-1) @ v[:, :, a:b])
    merged = merge_attention_partials(torch.stack(outs), torch.stack(lses))
    full = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    assert torch.allclose(merged, full, atol=1e-5, rtol=1e-5)
