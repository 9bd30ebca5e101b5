"""Tensor-parallel sharding (lowbit/tp.py) on CPU: the shard plan, bit-identical quantization of the shards, and the
row-parallel sum / vocabulary-parallel argmax over a world-size-2 gloo group."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from lowbit import quant, tp

ARCHS = {"3b": (16, 2, 128, 11008, 151936), "7b": (28, 4, 128, 18944, 152064), "0.5b": (14, 2, 64, 4864, 151936)}


@pytest.mark.parametrize("arch", list(ARCHS))
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_every_head_row_and_token_once(arch, world):
    nh, nkv, hd, inter, vocab = ARCHS[arch]
    try:
        plans = [tp.plan(nh, nkv, hd, inter, vocab, world, r) for r in range(world)]
    except ValueError:
        # only layouts the kernels cannot group uniformly are refused
        assert not (nkv % world == 0 or (world % nkv == 0 and world // nkv <= nh // nkv))
        return
    g = nh // nkv
    q = [h for p in plans for h in range(*p["q_heads"])]
    assert q == list(range(nh))
    for p in plans:
        k0, k1 = p["kv_heads"]
        local_q = range(*p["q_heads"])
        # one uniform group per local kv head: every local q head belongs to a local kv head
        assert all(k0 <= h // g < k1 for h in local_q)
        nq, nk = len(local_q), k1 - k0
        assert nq % nk == 0
        assert p["inter"][0] % tp.GROUP == 0 and p["inter"][1] % tp.GROUP == 0
    assert [r for p in plans for r in range(*p["inter"])] == list(range(inter))
    assert [r for p in plans for r in range(*p["vocab"])] == list(range(vocab))
    if world > nkv:   # the kv heads are replicated, each on world / nkv ranks
        assert sorted(p["kv_heads"][0] for p in plans) == sorted(list(range(nkv)) * (world // nkv))


def test_plan_refusals():
    with pytest.raises(ValueError):
        tp.plan(28, 4, 128, 18944, 152064, 3, 0)     # 4 kv heads over 3 ranks
    with pytest.raises(ValueError):
        tp.plan(28, 4, 128, 18944, 152064, 2, 2)     # rank out of range
    with pytest.raises(ValueError):
        tp.plan(28, 4, 128, 1000, 152064, 2, 0)      # intermediate not a multiple of 128
    with pytest.raises(ValueError):
        tp.plan(6, 4, 128, 1024, 100, 2, 0)          # heads do not group


def _layer(rng, h=256, inter=512, nh=4, nkv=2, hd=64):
    w = lambda o, i: torch.from_numpy((rng.standard_normal((o, i)) * 0.02).astype(np.float32))
    b = lambda o: torch.from_numpy((rng.standard_normal(o) * 0.02).astype(np.float32))
    return {"q": w(nh * hd, h), "k": w(nkv * hd, h), "v": w(nkv * hd, h), "o": w(h, nh * hd), "gate": w(inter, h),
            "up": w(inter, h), "down": w(h, inter), "q_b": b(nh * hd), "k_b": b(nkv * hd), "v_b": b(nkv * hd)}


@pytest.mark.parametrize("world", [2, 4])
def test_sharded_quantization_is_bit_identical(world):
    """Row-parallel shards split K on group boundaries, column-parallel shards split rows: every shard's packed
    bytes and scales are a slice of the unsharded quantization."""
    rng = np.random.default_rng(world)
    w = _layer(rng, inter=1024, nh=8, nkv=2)
    full = {k: quant.quantize_w4(w[k].numpy(), 128) for k in ("o", "down", "gate", "up", "q", "k", "v")}
    for r in range(world):
        p = tp.plan(8, 2, 64, 1024, 1000, world, r)
        sh = tp.shard_layer(w, p)
        i0, i1 = p["inter"]
        q0, q1 = p["q_heads"]
        pk, sc = quant.quantize_w4(sh["down"].numpy(), 128)
        assert np.array_equal(pk, full["down"][0][:, i0 // 2:i1 // 2])
        assert np.array_equal(sc.view(np.uint16), full["down"][1][:, i0 // 128:i1 // 128].view(np.uint16))
        pk, sc = quant.quantize_w4(sh["o"].numpy(), 128)
        if 64 * (q1 - q0) % 128 == 0:   # head pairs: whole groups of o's K
            assert np.array_equal(pk, full["o"][0][:, q0 * 32:q1 * 32])
        pk, _ = quant.quantize_w4(sh["gu"].numpy(), 128)
        assert np.array_equal(pk, np.concatenate([full["gate"][0][i0:i1], full["up"][0][i0:i1]]))
        pk, _ = quant.quantize_w4(tp.shard_layer(w, p, interleave=True)["gu"].numpy(), 128)
        assert np.array_equal(pk[0::2], full["gate"][0][i0:i1]) and np.array_equal(pk[1::2], full["up"][0][i0:i1])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        w = _layer(rng, inter=1024)
        x = torch.from_numpy(rng.standard_normal(256).astype(np.float32))
        p = tp.plan(4, 2, 64, 1024, 1000, world, rank)
        sh = tp.shard_layer(w, p)
        # row-parallel MLP partial on the dequantized shard weights, summed over ranks
        deq = lambda t: torch.from_numpy(quant.dequantize_w4(*quant.quantize_w4(t.numpy(), 128), 128))
        gu = deq(sh["gu"]) @ x
        i = gu.shape[0] // 2
        a = torch.nn.functional.silu(gu[:i]) * gu[i:]
        y = deq(sh["down"]) @ a
        dist.all_reduce(y)
        full = deq(w["down"]) @ (torch.nn.functional.silu(deq(w["gate"]) @ x) * (deq(w["up"]) @ x))
        results[f"mlp{rank}"] = float((y - full).abs().max() / full.abs().max())
        # vocabulary-parallel argmax with a tie spanning the two shards: the first occurrence wins
        logits = torch.zeros(1000)
        logits[[10, 700]] = 5.0
        v0, v1 = p["vocab"]
        val, idx = logits[v0:v1].max(-1)
        pair = torch.stack([val, (idx + v0).float()])
        pairs = torch.zeros(2 * world)
        dist.all_gather_into_tensor(pairs, pair)
        pr = pairs.view(world, 2)
        results[f"tok{rank}"] = int(pr[pr[:, 0].argmax(), 1])
    finally:
        dist.destroy_process_group()


def test_row_parallel_sum_and_vocab_argmax_over_gloo():
    world = 2
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn")
    for r in range(world):
        assert results[f"mlp{r}"] < 1e-5, results[f"mlp{r}"]
        assert results[f"tok{r}"] == 10


def _attn_worker(rank, world, port, results):
    """One rank of a tensor-parallel attention block at the Qwen2.5-7B head layout (28 query heads, 4 kv heads, so at
    8 ranks each kv head is held by two ranks that split its 7 query heads 3 + 4), small dims, fp64: the rank's
    q|k|v rows, grouped attention of its local heads over a cache, its o-projection partial, summed over ranks."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        nh, nkv, hd, inter, ctx = 28, 4, 16, 1024, 6
        h = nh * hd
        g = torch.Generator().manual_seed(21)
        w = {"q": torch.randn(nh * hd, h, generator=g, dtype=torch.float64) * 0.05,
             "k": torch.randn(nkv * hd, h, generator=g, dtype=torch.float64) * 0.05,
             "v": torch.randn(nkv * hd, h, generator=g, dtype=torch.float64) * 0.05,
             "o": torch.randn(h, nh * hd, generator=g, dtype=torch.float64) * 0.05,
             "gate": torch.randn(inter, h, generator=g, dtype=torch.float64),
             "up": torch.randn(inter, h, generator=g, dtype=torch.float64),
             "down": torch.randn(h, inter, generator=g, dtype=torch.float64),
             "q_b": torch.randn(nh * hd, generator=g, dtype=torch.float64) * 0.1,
             "k_b": torch.randn(nkv * hd, generator=g, dtype=torch.float64) * 0.1,
             "v_b": torch.randn(nkv * hd, generator=g, dtype=torch.float64) * 0.1}
        x = torch.randn(h, generator=g, dtype=torch.float64)
        kcache = torch.randn(nkv, ctx, hd, generator=g, dtype=torch.float64)
        vcache = torch.randn(nkv, ctx, hd, generator=g, dtype=torch.float64)

        def attend(q, k_new, v_new, kc, vc, n_q, n_kv):
            grp = n_q // n_kv
            out = []
            for i in range(n_q):
                j = i // grp                                   # one uniform query group per kv head
                K = torch.cat([kc[j], k_new[j][None]])
                V = torch.cat([vc[j], v_new[j][None]])
                a = torch.softmax(K @ q[i] / hd ** 0.5, 0)
                out.append(a @ V)
            return torch.cat(out)

        # unsharded reference
        qf = (w["q"] @ x + w["q_b"]).view(nh, hd)
        kf = (w["k"] @ x + w["k_b"]).view(nkv, hd)
        vf = (w["v"] @ x + w["v_b"]).view(nkv, hd)
        want = w["o"] @ attend(qf, kf, vf, kcache, vcache, nh, nkv)

        p = tp.plan(nh, nkv, hd, inter, 1000, world, rank)
        sh = tp.shard_layer(w, p)
        (q0, q1), (k0, k1) = p["q_heads"], p["kv_heads"]
        nq, nk = q1 - q0, k1 - k0
        qkv = sh["qkv"] @ x + sh["bias"]
        q = qkv[:nq * hd].view(nq, hd)
        k_new = qkv[nq * hd:(nq + nk) * hd].view(nk, hd)
        v_new = qkv[(nq + nk) * hd:].view(nk, hd)
        y = sh["o"] @ attend(q, k_new, v_new, kcache[k0:k1], vcache[k0:k1], nq, nk)
        dist.all_reduce(y)
        results[f"err{rank}"] = float((y - want).abs().max() / want.abs().max())
        results[f"heads{rank}"] = (nq, nk)
    finally:
        dist.destroy_process_group()


def test_uneven_tp8_attention_over_gloo():
    """Qwen2.5-7B's head layout split over 8 ranks (kv heads replicated, query groups 3 + 4) reproduces the
    unsharded attention block: shard plan, fused q|k|v rows and bias, local grouping, row-parallel o and the sum."""
    world = 8
    results = mp.get_context("spawn").Manager().dict()
    mp.start_processes(_attn_worker, args=(world, _free_port(), results), nprocs=world, start_method="spawn")
    assert sorted(results[f"heads{r}"] for r in range(world)) == [(3, 1)] * 4 + [(4, 1)] * 4
    for r in range(world):
        assert results[f"err{r}"] < 1e-12, results[f"err{r}"]
