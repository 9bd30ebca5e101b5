"""Tensor-parallel INT4 decode over NCCL (2 GPUs): the sharded decoder's tokens and logits against the single-GPU
decoder on the same weights. Skipped with fewer than two GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

TINY = dict(hidden_size=256, intermediate_size=640, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, vocab_size=1024, tie_word_embeddings=False)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, results, fuse=()):
    from datetime import timedelta
    import torch.distributed as dist
    from lowbit import decode
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        decode.enable_decode_options()
        gen = torch.Generator().manual_seed(1)
        prompt = torch.randint(0, TINY["vocab_size"], (20,), generator=gen)
        seq = torch.randint(0, TINY["vocab_size"], (10,), generator=gen).tolist()
        dec = decode.Int4Decoder(decode.build(TINY, seed=3, device=dev), 48, world=world, rank=rank,
                                 pg=dist.group.WORLD, fuse=fuse)
        dec.prefill(prompt)
        got = dec.forced(seq)
        toks = []
        dec.prefill(prompt)
        for _ in range(6):
            dec.step()
            toks.append(dec.tok.item())
        ref = decode.Int4Decoder(decode.build(TINY, seed=3, device=dev), 48)
        ref.prefill(prompt)
        want = ref.forced(seq)[:, dec.vocab0:dec.vocab0 + got.shape[1]]
        ref_toks = []
        ref.prefill(prompt)
        for _ in range(6):
            ref.step()
            ref_toks.append(ref.tok.item())
        results[f"err{rank}"] = float((got - want).abs().max() / want.pow(2).mean().sqrt())
        results[f"toks{rank}"] = (toks, ref_toks)
        dec.graph = None
        ref.graph = None
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fuse", [(), ("epilogue",), ("epilogue", "gemv_allreduce")])
def test_tp2_decoder_matches_single_gpu(fuse):
    """fuse=("epilogue",): the residual add + RMSNorm run inside the one-shot allreduce; + "gemv_allreduce": the o
    and down GEMVs push their tiles to every rank and sum, add and normalize in their last CTA"""
    world = 2
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_rank, args=(world, _free_port(), results, fuse), nprocs=world, start_method="spawn")
    for r in range(world):
        assert results[f"err{r}"] < 2e-2, results[f"err{r}"]
        toks, ref_toks = results[f"toks{r}"]
        assert sum(a == b for a, b in zip(toks, ref_toks)) >= 5, (toks, ref_toks)


def _ar_rank(rank, world, port, results):
    from datetime import timedelta
    import torch.distributed as dist
    from lowbit import ops, tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        ar = tp.OneShotAllReduce(3584, dist.group.WORLD, dev)
        ok = True
        for call in range(5):   # epochs cycle through both slots
            g = torch.Generator(device=dev).manual_seed(100 * call + rank)
            t = torch.randn(3584, device=dev, generator=g).half()
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            want = torch.stack(parts).float().sum(0).half()   # rank order, fp32, one rounding
            ar(t)
            torch.cuda.synchronize()
            ok = ok and torch.equal(t, want)
        # in a CUDA graph: replays advance the device epoch
        x = torch.ones(3584, device=dev).half() * (rank + 1)
        gph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            y = x.clone()
            ar(y)
        torch.cuda.current_stream().wait_stream(s)
        with torch.cuda.graph(gph):
            y = x.clone()
            ar(y)
        for _ in range(3):
            gph.replay()
        torch.cuda.synchronize()
        ok = ok and torch.all(y == sum(range(1, world + 1))).item()
        results[f"ok{rank}"] = bool(ok)
        results[f"err{rank}"] = ops.ext().lib.lb_device_error()
        del gph
        torch.cuda.synchronize()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_oneshot_allreduce_matches_rank_ordered_sum():
    world = 2
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_ar_rank, args=(world, _free_port(), results), nprocs=world, start_method="spawn")
    for r in range(world):
        assert results[f"ok{r}"] and results[f"err{r}"] == 0
