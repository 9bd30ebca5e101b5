"""Tensor-parallel sharding of a Qwen2 decoder for INT4 decode (the benchmark's multi-GPU config).

Column-parallel q|k|v (by attention heads) and gate|up (by 128-row groups of the intermediate size), row-parallel
o and down on the matching 128-column groups -- so every shard's INT4 groups are exactly the unsharded model's and
the quantized bits are identical -- each followed by one sum allreduce, and a vocabulary-parallel lm_head (local
argmax, then an all-gather of (value, index) pairs). The reference has no multi-GPU code; this follows its
layer math (lowbit/model.py:15-27 applied to each shard).

Attention heads: with world <= kv heads each rank takes whole kv heads and their query groups; with more ranks
than kv heads (Qwen2.5-7B at 8 GPUs: 4 kv heads, 28 query heads), the ranks sharing a kv head each hold a copy of
it and split its query group (7 heads -> 4 + 3), so every rank keeps one uniform query group per local kv head.
"""
GROUP = 128


def even_split(n, parts):
    """[(start, stop)] of `parts` contiguous ranges covering range(n), sizes differing by at most one."""
    return [(n * i // parts, n * (i + 1) // parts) for i in range(parts)]


def plan(nh, nkv, hd, inter, vocab, world, rank):
    """The shard of `rank`: global q heads, kv heads, intermediate rows (128-aligned) and vocabulary rows."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if nh % nkv:
        raise ValueError(f"{nh} query heads do not group over {nkv} kv heads")
    g = nh // nkv
    if world <= nkv:
        if nkv % world:
            raise ValueError(f"{nkv} kv heads do not divide over {world} ranks")
        per = nkv // world
        kv = (rank * per, (rank + 1) * per)
        q = (kv[0] * g, kv[1] * g)
    else:
        if world % nkv:
            raise ValueError(f"{world} ranks do not divide over {nkv} kv heads")
        share = world // nkv
        if share > g:
            raise ValueError(f"{share} ranks per kv head but only {g} query heads each")
        head = rank // share
        lo, hi = even_split(g, share)[rank % share]
        kv = (head, head + 1)
        q = (head * g + lo, head * g + hi)
    if inter % GROUP:
        raise ValueError(f"intermediate size {inter} is not a multiple of {GROUP}")
    gl, gh = even_split(inter // GROUP, world)[rank]
    return {"q_heads": q, "kv_heads": kv, "inter": (gl * GROUP, gh * GROUP),
            "vocab": even_split(vocab, world)[rank], "hd": hd}


def shard_layer(w, p, interleave=False):
    """Slice one decoder layer's fp16 weights (dict of torch tensors: q, k, v, o, gate, up, down weights and
    q_b, k_b, v_b biases, nn.Linear [out, in] layout) to the shard `p`. Returns the fused q|k|v rows (+ bias),
    the o columns, the fused gate|up rows -- [gate; up], or with `interleave` gate_0, up_0, gate_1, up_1, ...
    (the layout of the SwiGLU-epilogue GEMV) -- and the down columns. Quantization is per row, so either order
    holds the same quantized rows."""
    import torch
    hd = p["hd"]
    q0, q1 = p["q_heads"]
    k0, k1 = p["kv_heads"]
    i0, i1 = p["inter"]
    qr, kr = slice(q0 * hd, q1 * hd), slice(k0 * hd, k1 * hd)
    qkv = torch.cat([w["q"][qr], w["k"][kr], w["v"][kr]], 0)
    bias = None if w.get("q_b") is None else torch.cat([w["q_b"][qr], w["k_b"][kr], w["v_b"][kr]], 0)
    return {"qkv": qkv.contiguous(), "bias": bias,
            "o": w["o"][:, qr].contiguous(),
            "gu": (torch.stack([w["gate"][i0:i1], w["up"][i0:i1]], 1).reshape(2 * (i1 - i0), -1) if interleave
                   else torch.cat([w["gate"][i0:i1], w["up"][i0:i1]], 0)).contiguous(),
            "down": w["down"][:, i0:i1].contiguous()}


class OneShotAllReduce:
    """In-place sum allreduce of small fp16 tensors for tensor-parallel decode: the library's one-shot kernel
    (lb_tp_allreduce: one launch per call on each rank, peer loads over NVLink, bounded waits) on peer-mapped
    buffers that torch's symmetric memory allocates and exchanges (plumbing only). The same allocation holds a
    second region for the row-parallel GEMV fused with the allreduce (lb_tp_gemv_allreduce_norm), which pushes
    each finished tile into every rank's region and has its own epoch."""

    FLAG_BYTES = 256

    def __init__(self, cap, group, device):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm
        from . import ops
        self.lib = ops.ext().lib
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if self.world > 64:
            raise ValueError("at most 64 ranks")
        self.cap = (cap + 7) // 8 * 8
        try:
            symm.enable_symm_mem_for_group(group.group_name)
        except Exception:   # noqa: BLE001 - newer torch enables groups on first use
            pass
        pull = self.FLAG_BYTES // 2 + 2 * self.cap                  # halves: flags + 2 slots
        push = self.FLAG_BYTES // 2 + 4 * self.world * self.cap      # header + 2 x world regions of cap / 2 words
        self.buf = symm.empty(pull + push, dtype=torch.half, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        handle = symm.rendezvous(self.buf, group)
        off = self.buf.data_ptr() - handle.buffer_ptrs[self.rank]
        self.ptrs = torch.tensor([p + off for p in handle.buffer_ptrs], dtype=torch.int64, device=device)
        self.push_ptrs = self.ptrs + 2 * pull
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.push_epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.handle = handle
        dist.barrier(group)

    def __call__(self, t):
        import torch
        rc = self.lib.lb_tp_allreduce(t.data_ptr(), t.data_ptr(), t.numel(), self.cap, self.ptrs.data_ptr(),
                                      self.epoch.data_ptr(), self.rank, self.world,
                                      torch.cuda.current_stream(t.device).cuda_stream)
        if rc:
            raise RuntimeError(self.lib.lb_last_error().decode())
        return t

    def gemv_residual_norm(self, x, wq, x_res, norm_w, h, eps, counter):
        """One kernel: this rank's row-parallel GEMV partial W x, summed over the ranks, added into x_res; h =
        RMSNorm(x_res) * norm_w (lb_tp_gemv_allreduce_norm). counter: a zeroed device int32 of this call site."""
        import torch
        rc = self.lib.lb_tp_gemv_allreduce_norm(
            x.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(), None, wq.n, wq.k, wq.group, self.cap,
            self.push_ptrs.data_ptr(), self.push_epoch.data_ptr(), self.rank, self.world, x_res.data_ptr(),
            norm_w.data_ptr(), h.data_ptr(), eps, counter.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream)
        if rc:
            raise RuntimeError(self.lib.lb_last_error().decode())

    def residual_norm(self, t, x_res, norm_w, h, eps):
        """x_res += the sum of every rank's t; h = RMSNorm(x_res) * norm_w (lb_tp_allreduce_norm, one launch);
        t is left as it was."""
        import torch
        rc = self.lib.lb_tp_allreduce_norm(t.data_ptr(), t.numel(), self.cap, self.ptrs.data_ptr(),
                                           self.epoch.data_ptr(), self.rank, self.world, x_res.data_ptr(),
                                           norm_w.data_ptr(), h.data_ptr(), eps,
                                           torch.cuda.current_stream(t.device).cuda_stream)
        if rc:
            raise RuntimeError(self.lib.lb_last_error().decode())
