"""Batch-1 greedy decode of a random-init Qwen2.5-architecture decoder through the INT4 kernels.

The measurement of the reference's bench/e2e.py (`speed_graph`, bench/e2e.py:84-147) -- every decode step (one token
through all layers, the lm_head and the argmax) captured as one CUDA graph over a static KV cache and replayed --
without checkpoint or dataset: weights come from the transformers Qwen2 initializer (N(0, 0.02)) and prompt ids are
uniform over the vocabulary, so the bytes moved per token are those of the real model.

`Int4Decoder` is the product path: the model's projections quantized once (q|k|v and gate|up fused row-wise into
one INT4 weight each: rows quantize independently, so the bits equal the separate layers'), the decode-step kernels
of the library around the INT4 GEMVs, and position / token in device memory so a graph replays every step.
`GraphDecoder` (transformers forward + W4Linear, as the reference runs it) is kept for comparison; with
transformers 5.5 a captured transformers step replays wrong logits for the fp16 model too, so it is not timed.
"""
import torch

from . import model as lbm
from . import ops, tp

# Qwen2.5 architectures of the benchmark configs (head_dim 128, RMSNorm eps 1e-6, RoPE theta 1e6, SwiGLU)
QWEN25_3B = dict(hidden_size=2048, intermediate_size=11008, num_hidden_layers=36, num_attention_heads=16,
                 num_key_value_heads=2, vocab_size=151936, tie_word_embeddings=True)
QWEN25_7B = dict(hidden_size=3584, intermediate_size=18944, num_hidden_layers=28, num_attention_heads=28,
                 num_key_value_heads=4, vocab_size=152064, tie_word_embeddings=False)


def qwen2_config(arch, **overrides):
    from transformers import Qwen2Config
    kw = dict(arch, rms_norm_eps=1e-6, max_position_embeddings=32768,
              rope_parameters={"rope_type": "default", "rope_theta": 1e6})
    kw.update(overrides)
    cfg = Qwen2Config(**kw)
    cfg._attn_implementation = "sdpa"
    return cfg


@torch.no_grad()
def build(arch, seed=0, device="cuda", **overrides):
    """A random-init fp16 Qwen2ForCausalLM, initialized directly on `device`."""
    from transformers import Qwen2ForCausalLM
    cfg = qwen2_config(arch, **overrides)
    torch.manual_seed(seed)
    with torch.device(device):
        m = Qwen2ForCausalLM(cfg)
    return m.half().eval()


def to_int4(model, group=128):
    """Quantize every decoder projection on the GPU and swap in W4Linear; returns (layers, INT4 bytes)."""
    return lbm.apply_int4(lbm.quantize_layers(model, group), group)


def to_fake_quant(model, group=128):
    """The same quantized values as fp16 nn.Linear weights (cuBLAS on the dequantized weights)."""
    lbm.apply_fake_quant(lbm.quantize_layers(model, group), group)
    return model


def bytes_per_token(model, context, int4_bytes):
    """HBM bytes one decode step must read: INT4 projections + fp16 lm_head + the KV cache at `context`."""
    cfg = model.config
    head = model.lm_head.weight.numel() * 2
    kv = 2 * cfg.num_hidden_layers * cfg.num_key_value_heads * (cfg.hidden_size // cfg.num_attention_heads) * 2 * context
    return int4_bytes + head + kv


class GraphDecoder:
    """Static-cache greedy decoding, one CUDA graph per step (bench/e2e.py:84-147). The token fed and its cache
    position live in static device tensors that the step itself advances, so replays need no host work."""

    def __init__(self, model, max_len):
        from transformers import StaticCache
        self.model, self.max_len = model, max_len
        self.cache = StaticCache(config=model.config, max_cache_len=max_len)
        dev = model.model.embed_tokens.weight.device
        self.tok = torch.zeros(1, 1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.logits = None
        self.graph = None

    def _step(self):
        out = self.model(input_ids=self.tok, past_key_values=self.cache, cache_position=self.pos, use_cache=True)
        self.logits = out.logits[:, -1]
        self.tok.copy_(self.logits.argmax(-1, keepdim=True))
        self.pos.add_(1)

    @torch.no_grad()
    def prefill(self, ids):
        """Run the prompt [1, p] eagerly into the cache; the next token to feed is its greedy continuation."""
        self.cache.reset()
        p = ids.shape[1]
        out = self.model(input_ids=ids, past_key_values=self.cache,
                         cache_position=torch.arange(p, device=ids.device), use_cache=True)
        self.tok.copy_(out.logits[:, -1].argmax(-1, keepdim=True))
        self.pos.fill_(p)
        return out.logits[0, -1]

    @torch.no_grad()
    def capture(self):
        """Warm the step up on a side stream, then capture it. Warm-up writes cache slots that the real steps
        overwrite, and the token / position are restored."""
        tok, pos = self.tok.clone(), self.pos.clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step()
        torch.cuda.current_stream().wait_stream(s)
        self.tok.copy_(tok)
        self.pos.copy_(pos)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step()
        self.graph = g
        self.tok.copy_(tok)
        self.pos.copy_(pos)
        torch.cuda.synchronize()

    def step(self):
        self.graph.replay()

    @torch.no_grad()
    def forced(self, seq):
        """Logits of the graph step for each token of `seq` fed in turn (teacher forcing), float32 [len, vocab]."""
        rows = []
        for t in seq:
            self.tok.fill_(int(t))
            self.graph.replay()
            rows.append(self.logits[0].float().clone())
        return torch.stack(rows)


def enable_decode_options():
    """PDL chaining between the library's kernels, weights fetched before the stream dependency (they are static
    model state)."""
    e = ops.ext()
    e.set_option("pdl", 1)
    e.set_option("early_weights", 1)


class Int4Decoder:
    """Qwen2 decode step on the library's kernels: embed -> per layer [RMSNorm + q|k|v GEMV, attention (bias +
    RoPE + KV append + split attention, combine), o GEMV, residual + RMSNorm + gate|up GEMV, SiLU*up + down GEMV]
    -> final RMSNorm -> fp16 lm_head (cuBLAS) -> argmax. Takes the weights of a transformers Qwen2ForCausalLM
    (fp16, nn.Linear projections) and frees its decoder layers.

    `fuse` picks kernel fusions: "norm_epilogue" ends the o and down GEMVs with the residual add + next RMSNorm
    (the last CTA of the GEMV, or the one-shot allreduce under tensor parallelism); "swiglu_epilogue" ends the
    gate|up GEMV with SiLU*up (its rows interleaved); "epilogue" is both, so a layer is q|k|v GEMV, attention, o,
    gate|up, down; under tensor parallelism with the one-shot allreduce, "gemv_allreduce" also fuses the o and down
    GEMVs with their allreduce (each finished tile pushed over NVLink into every rank's buffer, the last CTA
    summing and normalizing: one kernel instead of two). "qkv", "gu", "down" instead fold the preceding norm or
    SwiGLU into the GEMV's prologue where one CTA holds the row."""

    def __init__(self, model, max_len, group=128, world=1, rank=0, pg=None, fuse=(), allreduce="oneshot"):
        e = ops.ext()
        self.lib = e.lib
        cfg = model.config
        self.H, I = cfg.hidden_size, cfg.intermediate_size
        nh, nkv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.hd = self.H // nh
        self.eps = float(cfg.rms_norm_eps)
        self.max_len = max_len
        self.world, self.rank, self.pg = world, rank, pg
        self.gemv_ar = world > 1 and allreduce == "oneshot" and "gemv_allreduce" in fuse
        self.epi_norm = "epilogue" in fuse or "norm_epilogue" in fuse or self.gemv_ar
        self.epi_swiglu = "epilogue" in fuse or "swiglu_epilogue" in fuse
        self.epilogue = self.epi_norm or self.epi_swiglu
        theta = float(cfg.rope_parameters["rope_theta"])
        dev = model.model.embed_tokens.weight.device
        self.device = dev
        hd = self.hd
        shard = tp.plan(nh, nkv, hd, I, cfg.vocab_size, world, rank)
        self.nh = shard["q_heads"][1] - shard["q_heads"][0]
        self.nkv = shard["kv_heads"][1] - shard["kv_heads"][0]
        self.I = shard["inter"][1] - shard["inter"][0]
        self.vocab0 = shard["vocab"][0]

        def w4(weight):
            packed, scales = ops.quantize_w4_gpu(weight, group)
            return ops.W4Weight(packed, scales, group, ("mma",))

        self.layers, self.int4_bytes = [], 0
        with torch.no_grad():
            for layer in model.model.layers:
                a, m = layer.self_attn, layer.mlp
                w = {"q": a.q_proj.weight, "k": a.k_proj.weight, "v": a.v_proj.weight, "o": a.o_proj.weight,
                     "gate": m.gate_proj.weight, "up": m.up_proj.weight, "down": m.down_proj.weight,
                     "q_b": a.q_proj.bias, "k_b": a.k_proj.bias, "v_b": a.v_proj.bias}
                sh = tp.shard_layer(w, shard, interleave=self.epi_swiglu)
                ly = {
                    "qkv": w4(sh["qkv"]),
                    "bias": None if sh["bias"] is None else sh["bias"].half().contiguous(),
                    "o": w4(sh["o"]),
                    "gu": w4(sh["gu"]),
                    "down": w4(sh["down"]),
                    "ln1": layer.input_layernorm.weight.detach().half().contiguous(),
                    "ln2": layer.post_attention_layernorm.weight.detach().half().contiguous(),
                    "k": torch.zeros(self.nkv, max_len, hd, dtype=torch.half, device=dev),
                    "v": torch.zeros(self.nkv, max_len, hd, dtype=torch.half, device=dev),
                }
                self.int4_bytes += sum(ly[k].nbytes() for k in ("qkv", "o", "gu", "down"))
                # RMSNorm / SwiGLU folded into the GEMV that consumes them (`fuse`: which of q|k|v, gate|up, down)
                # where one CTA holds the whole row. Off by default: measured on B200 (3B, batch 1, 512 context) every
                # fusion is slower than the separate kernels (625 tok/s none, 598 q|k|v, 552 q|k|v + gate|up, 537
                # all): each of the GEMV's CTAs redoes the row's work (1376 CTAs for gate|up), which costs more
                # than one small launch under programmatic dependent launch
                for kind in ("qkv", "gu", "down"):
                    ly["fuse_" + kind] = (not self.epilogue and kind in fuse
                                          and bool(self.lib.lb_decode_gemv_fusable(ly[kind].n, ly[kind].k)))
                self.layers.append(ly)
        model.model.layers = None          # the fp16 projections are no longer needed
        torch.cuda.empty_cache()
        self.embed = model.model.embed_tokens.weight.detach()
        v0, v1 = shard["vocab"]
        self.head = model.lm_head.weight.detach()[v0:v1].contiguous() if world > 1 else model.lm_head.weight.detach()
        self.norm = model.model.norm.weight.detach().half().contiguous()
        self.inv_freq = (1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))).to(dev)
        self.tok = torch.zeros(1, dtype=torch.long, device=dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=dev)
        self.x = torch.zeros(self.H, dtype=torch.half, device=dev)     # residual stream (two buffers: a fused
        self.x2 = torch.zeros(self.H, dtype=torch.half, device=dev)    # norm GEMV writes x + r to the other)
        self.h = torch.zeros(self.H, dtype=torch.half, device=dev)
        self.attn = torch.zeros(1, self.nh * hd, dtype=torch.half, device=dev)
        self.act = torch.zeros(1, self.I, dtype=torch.half, device=dev)
        self.counters = torch.zeros(2, dtype=torch.int32, device=dev)   # last-CTA counters of the o, down GEMVs
        self.pair = torch.zeros(2, dtype=torch.float32, device=dev)
        self.pairs = torch.zeros(2 * world, dtype=torch.float32, device=dev)
        splits = self.lib.lb_decode_attention_splits(max_len)
        self.part_o = torch.zeros(self.nh * splits * hd, dtype=torch.float32, device=dev)
        self.part_ml = torch.zeros(self.nh * splits * 2, dtype=torch.float32, device=dev)
        self.logits = None
        self.graph = None
        # row-parallel sums: the library's one-shot kernel over peer memory, or NCCL
        self.allreduce = None
        if world > 1:
            if allreduce == "oneshot":
                self.allreduce = tp.OneShotAllReduce(self.H, pg, dev)
            else:
                self.allreduce = lambda t: torch.distributed.all_reduce(t, group=pg)

    def _ok(self, rc):
        if rc:
            raise RuntimeError(self.lib.lb_last_error().decode())

    def head_bytes(self):
        """fp16 lm_head bytes this rank reads per step (its vocabulary rows)."""
        return self.head.numel() * 2

    def kv_bytes(self, context):
        """KV-cache bytes this rank reads per step at `context` cached tokens."""
        return 2 * len(self.layers) * self.nkv * self.hd * 2 * context

    def _norm_gemv(self, x, r, ln, x_out, wq, st):
        y = torch.empty(1, wq.n, dtype=torch.half, device=self.device)
        self._ok(self.lib.lb_decode_norm_gemv(x.data_ptr(), None if r is None else r.data_ptr(), ln.data_ptr(),
                                              None if x_out is None else x_out.data_ptr(), self.eps,
                                              wq.packed_mma.data_ptr(), wq.scales.data_ptr(), y.data_ptr(), wq.n, wq.k,
                                              wq.group, st))
        return y

    def _residual_gemv(self, x, wq, ln, slot, st):
        """y = W x (row-parallel under tensor parallelism: summed over the ranks), then the residual stream
        self.x += y and self.h = RMSNorm(self.x) * ln -- in the GEMV's or the allreduce's epilogue with
        "norm_epilogue", else by the RMSNorm kernel."""
        y = torch.empty(1, wq.n, dtype=torch.half, device=self.device)
        if self.world == 1 and self.epi_norm:
            self._ok(self.lib.lb_decode_gemv_residual_norm(
                x.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(), y.data_ptr(), wq.n, wq.k, wq.group,
                self.x.data_ptr(), ln.data_ptr(), self.h.data_ptr(), self.eps, self.counters.data_ptr() + 4 * slot,
                st))
            return
        if self.gemv_ar:
            self.allreduce.gemv_residual_norm(x, wq, self.x, ln, self.h, self.eps, self.counters[slot:slot + 1])
            return
        y = ops.gemv(x, wq, 6)
        if self.epi_norm and isinstance(self.allreduce, tp.OneShotAllReduce):
            self.allreduce.residual_norm(y, self.x, ln, self.h, self.eps)
        else:
            if self.world > 1:
                self.allreduce(y)
            self._ok(self.lib.lb_decode_rmsnorm(self.x.data_ptr(), y.data_ptr(), ln.data_ptr(), self.h.data_ptr(),
                                                self.H, self.eps, st))

    def _step_epilogue(self):
        L, st = self.lib, torch.cuda.current_stream(self.device).cuda_stream
        nh, nkv, hd, H = self.nh, self.nkv, self.hd, self.H
        self._ok(L.lb_decode_embed(self.embed.data_ptr(), self.tok.data_ptr(), self.x.data_ptr(), H, st))
        self._ok(L.lb_decode_rmsnorm(self.x.data_ptr(), None, self.layers[0]["ln1"].data_ptr(), self.h.data_ptr(), H,
                                     self.eps, st))
        h2 = self.h.view(1, H)
        for i, ly in enumerate(self.layers):
            qkv = ops.gemv(h2, ly["qkv"], 6)
            self._ok(L.lb_decode_attention(qkv.data_ptr(), None if ly["bias"] is None else ly["bias"].data_ptr(),
                                           self.inv_freq.data_ptr(), self.pos.data_ptr(), ly["k"].data_ptr(),
                                           ly["v"].data_ptr(), self.part_o.data_ptr(), self.part_ml.data_ptr(),
                                           self.attn.data_ptr(), nh, nkv, hd, self.max_len, st))
            self._residual_gemv(self.attn, ly["o"], ly["ln2"], 0, st)
            wq = ly["gu"]
            if self.epi_swiglu:
                self._ok(L.lb_decode_gemv_swiglu(self.h.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(),
                                                 self.act.data_ptr(), wq.n, wq.k, wq.group, st))
            else:
                gu = ops.gemv(h2, wq, 6)
                self._ok(L.lb_decode_silu_mul(gu.data_ptr(), self.act.data_ptr(), self.I, st))
            nxt = self.layers[i + 1]["ln1"] if i + 1 < len(self.layers) else self.norm
            self._residual_gemv(self.act, ly["down"], nxt, 1, st)
        self._head()

    def _head(self):
        h2 = self.h.view(1, self.H)
        self.logits = torch.nn.functional.linear(h2, self.head)
        if self.world == 1:
            self.tok.copy_(self.logits.argmax(-1))
        else:
            # vocabulary-parallel argmax: each rank's best (value, global index); the first rank holding the
            # overall maximum wins, which is the first occurrence over the whole vocabulary
            val, idx = self.logits.float().max(-1)
            self.pair.copy_(torch.cat([val, (idx + self.vocab0).float()]))
            torch.distributed.all_gather_into_tensor(self.pairs, self.pair, group=self.pg)
            pr = self.pairs.view(self.world, 2)
            self.tok.copy_(pr[:, 1].gather(0, pr[:, 0].argmax().view(1)).long())   # no host sync
        self.pos.add_(1)

    def _step(self):
        if self.epilogue:
            return self._step_epilogue()
        L, st = self.lib, torch.cuda.current_stream(self.device).cuda_stream
        nh, nkv, hd, H = self.nh, self.nkv, self.hd, self.H
        cur, other = self.x, self.x2
        self._ok(L.lb_decode_embed(self.embed.data_ptr(), self.tok.data_ptr(), cur.data_ptr(), H, st))
        h2 = self.h.view(1, H)
        resid = None
        for ly in self.layers:
            if ly["fuse_qkv"]:
                qkv = self._norm_gemv(cur, resid, ly["ln1"], None if resid is None else other, ly["qkv"], st)
                if resid is not None:
                    cur, other = other, cur
            else:
                self._ok(L.lb_decode_rmsnorm(cur.data_ptr(), None if resid is None else resid.data_ptr(),
                                             ly["ln1"].data_ptr(), self.h.data_ptr(), H, self.eps, st))
                qkv = ops.gemv(h2, ly["qkv"], 6)
            self._ok(L.lb_decode_attention(qkv.data_ptr(), None if ly["bias"] is None else ly["bias"].data_ptr(),
                                           self.inv_freq.data_ptr(), self.pos.data_ptr(), ly["k"].data_ptr(),
                                           ly["v"].data_ptr(), self.part_o.data_ptr(), self.part_ml.data_ptr(),
                                           self.attn.data_ptr(), nh, nkv, hd, self.max_len, st))
            o = ops.gemv(self.attn, ly["o"], 6)
            if self.world > 1:
                self.allreduce(o)
            if ly["fuse_gu"]:
                gu = self._norm_gemv(cur, o, ly["ln2"], other, ly["gu"], st)
                cur, other = other, cur
            else:
                self._ok(L.lb_decode_rmsnorm(cur.data_ptr(), o.data_ptr(), ly["ln2"].data_ptr(), self.h.data_ptr(), H,
                                             self.eps, st))
                gu = ops.gemv(h2, ly["gu"], 6)
            if ly["fuse_down"]:
                wq = ly["down"]
                d = torch.empty(1, wq.n, dtype=torch.half, device=self.device)
                self._ok(L.lb_decode_swiglu_gemv(gu.data_ptr(), wq.packed_mma.data_ptr(), wq.scales.data_ptr(),
                                                 d.data_ptr(), wq.n, wq.k, wq.group, st))
            else:
                self._ok(L.lb_decode_silu_mul(gu.data_ptr(), self.act.data_ptr(), self.I, st))
                d = ops.gemv(self.act, ly["down"], 6)
            if self.world > 1:
                self.allreduce(d)
            resid = d
        self._ok(L.lb_decode_rmsnorm(cur.data_ptr(), None if resid is None else resid.data_ptr(),
                                     self.norm.data_ptr(), self.h.data_ptr(), H, self.eps, st))
        self._head()

    def launches_per_step(self):
        """Kernels of this library per step (the lm_head GEMV, the argmax and NCCL are not counted)."""
        oneshot = 2 * isinstance(self.allreduce, tp.OneShotAllReduce)   # the o and down allreduces of a layer
        if self.epilogue:   # q|k|v, attention (2), o, gate|up, down + the unfused norms and SiLU*up
            norms = 0 if self.epi_norm and (self.world == 1 or oneshot) else 2
            ar = oneshot if self.world > 1 and not self.gemv_ar else 0
            per = 6 + ar + norms + (not self.epi_swiglu)
            return 2 + per * len(self.layers)
        per = sum(6 + oneshot + (not ly["fuse_qkv"]) + (not ly["fuse_gu"]) + (not ly["fuse_down"])
                  for ly in self.layers)
        return 1 + per + 1

    @torch.no_grad()
    def capture(self):
        """Capture the step (after a warm-up on a side stream; token, position and cache row are restored)."""
        tok, pos = self.tok.clone(), self.pos.clone()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self._step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.tok.copy_(tok)
        self.pos.copy_(pos)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step()
        self.graph = g
        self.tok.copy_(tok)
        self.pos.copy_(pos)
        torch.cuda.synchronize(self.device)

    def step(self):
        self.graph.replay()

    @torch.no_grad()
    def prefill(self, ids):
        """Feed the prompt one token per graph step (ids: 1-D or [1, p]); the next token is its greedy
        continuation. Returns the last prompt token's logits."""
        ids = ids.reshape(-1).tolist()
        self.pos.fill_(0)
        if self.graph is None:
            self.capture()
        for t in ids:
            self.tok.fill_(int(t))
            self.graph.replay()
        return self.logits[0]

    @torch.no_grad()
    def forced(self, seq):
        """Logits after each token of `seq` fed in turn (teacher forcing), float32 [len, vocab]."""
        rows = []
        for t in seq:
            self.tok.fill_(int(t))
            self.graph.replay()
            rows.append(self.logits[0].float().clone())
        return torch.stack(rows)
