"""Two-GPU check of the row-sharded block (skipped with fewer than two GPUs):
head-parallel video self-attention (Q/K/V all-to-all), the split-key
video->audio attention merged by log-sum-exp, and the side-stream
exchanges, against the same blocks run unsharded on one GPU."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _build(dev, batch=1):
    from ltxq.block import BasicAVTransformerBlock, StreamConfig, TransformerArgs

    video = StreamConfig(1024, 8, 128, 1024)
    audio = StreamConfig(512, 8, 64, 512)
    gen = torch.Generator(device=dev)
    gen.manual_seed(90)  # identical on every rank
    blocks = [BasicAVTransformerBlock.random(gen, dev, mode="mxfp8", video=video, audio=audio) for _ in range(2)]

    def rnd(*shape, std=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=gen, device=dev) * std).to(dtype)

    def rope(heads, t, d):
        ang = torch.rand(1, heads, t, d // 2, generator=gen, device=dev) * 6.28
        return torch.cos(ang), torch.sin(ang)

    T, A, L, B = 128, 40, 32, batch  # batch 2: the CFG pair as one pass, per-batch AdaLN vectors
    v = TransformerArgs(x=rnd(B, T, video.dim, dtype=torch.bfloat16), context=rnd(B, L, video.context_dim,
                                                                                   dtype=torch.bfloat16),
                        timesteps=rnd(B, 1, 9, video.dim, std=0.1), positional_embeddings=rope(video.heads, T, 128),
                        cross_positional_embeddings=rope(audio.heads, T, 64),
                        cross_scale_shift_timestep=rnd(B, 1, 4, video.dim, std=0.1),
                        cross_gate_timestep=rnd(B, 1, 1, video.dim, std=0.1),
                        prompt_timestep=rnd(B, 1, 2, video.dim, std=0.1))
    a = TransformerArgs(x=rnd(B, A, audio.dim, dtype=torch.bfloat16), context=rnd(B, L, audio.context_dim,
                                                                                   dtype=torch.bfloat16),
                        timesteps=rnd(B, 1, 9, audio.dim, std=0.1), positional_embeddings=rope(audio.heads, A, 64),
                        cross_positional_embeddings=rope(audio.heads, A, 64),
                        cross_scale_shift_timestep=rnd(B, 1, 4, audio.dim, std=0.1),
                        cross_gate_timestep=rnd(B, 1, 1, audio.dim, std=0.1),
                        prompt_timestep=rnd(B, 1, 2, audio.dim, std=0.1))
    return blocks, v, a


def _rows(args, lo, hi):
    return args.replace(x=args.x[:, lo:hi].contiguous(),
                        positional_embeddings=tuple(c[:, :, lo:hi].contiguous() for c in args.positional_embeddings),
                        cross_positional_embeddings=tuple(c[:, :, lo:hi].contiguous()
                                                          for c in args.cross_positional_embeddings))


def _worker(rank, world, port, out_dir, self_attention, v2a, batch):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "ltx-2-mlx_b200")]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    from ltxq.block import RowShard

    blocks, v, a = _build(dev, batch)
    T = v.x.shape[1]
    tl = T // world
    shard = RowShard(dist.group.WORLD, world, rank, self_attention=self_attention, v2a=v2a)
    vv, aa = _rows(v, rank * tl, (rank + 1) * tl), a
    for b in blocks:
        vv, aa = b(vv, aa, shard)
    torch.cuda.synchronize()
    torch.save({"v": vv.x.cpu(), "a": aa.x.cpu()}, os.path.join(out_dir, f"r{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("self_attention,v2a,batch", [("gather", "gather", 1), ("head_parallel", "split_keys", 1),
                                                       ("gather", "gather", 2), ("head_parallel", "split_keys", 2)])
def test_row_sharded_block_matches_unsharded(cuda, tmp_path, self_attention, v2a, batch):
    world = 2
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path), self_attention, v2a, batch), nprocs=world,
                       join=True, start_method="spawn")
    from oracle import ref_ops as ro

    blocks, v, a = _build(torch.device("cuda", 0), batch)
    for b in blocks:
        v, a = b(v, a)
    got_v = torch.cat([torch.load(os.path.join(tmp_path, f"r{r}.pt"))["v"] for r in range(world)], dim=1)
    got_a = [torch.load(os.path.join(tmp_path, f"r{r}.pt"))["a"] for r in range(world)]
    ref_v, ref_a = v.x.cpu().float().numpy(), a.x.cpu().float().numpy()
    for got, ref, what in ((got_v.float().numpy(), ref_v, "video"), (got_a[0].float().numpy(), ref_a, "audio"),
                           (got_a[1].float().numpy(), ref_a, "audio rank 1")):
        mar, cos = ro.max_abs_rel(got, ref), ro.cosine(got, ref)
        assert mar <= 2e-2 and cos >= 0.9995, f"{what}: max_abs_rel={mar:.3e} cos={cos:.6f}"
