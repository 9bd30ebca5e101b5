"""The decode harness (random-init Qwen2 decoder, INT4 projections, one CUDA graph per step) on a small config.

The INT4 model is compared with the fake-quant model -- the same quantized values as fp16 nn.Linear weights run
through cuBLAS (the split the reference's bench/e2e.py uses to isolate kernel error from quantization error).
"""
import pytest
import torch

from lowbit import decode, ops

pytestmark = pytest.mark.gpu

TINY = dict(hidden_size=256, intermediate_size=640, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, vocab_size=1024, tie_word_embeddings=True)


@torch.no_grad()
def test_int4_decoder_matches_fake_quant_and_replays_bit_exactly():
    decode.enable_decode_options()
    gen = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, TINY["vocab_size"], (24,), generator=gen)
    seq = torch.randint(0, TINY["vocab_size"], (12,), generator=gen).tolist()

    dec = decode.Int4Decoder(decode.build(TINY, seed=3), max_len=64)
    assert dec.int4_bytes > 0
    first = dec.prefill(prompt).float()
    got = dec.forced(seq)

    f = decode.to_fake_quant(decode.build(TINY, seed=3))
    full = torch.cat([prompt, torch.tensor(seq)]).view(1, -1).cuda()
    want = f(input_ids=full).logits[0].float()
    p = prompt.numel()
    want_first, want_rows = want[p - 1], want[p:]
    rms = want_rows.pow(2).mean().sqrt()
    err = (got - want_rows).abs().max() / rms
    assert err < 2e-2, f"normalized logit error {err:.3e}"
    assert ((first - want_first).abs().max() / rms) < 2e-2
    agree = (got.argmax(-1) == want_rows.argmax(-1)).float().mean().item()
    assert agree >= 0.9, agree

    # a graph replay is the eager step, bit for bit
    for run in ("graph", "eager"):
        dec.pos.fill_(p)
        dec.tok.fill_(seq[0])
        if run == "graph":
            dec.graph.replay()
            replay = dec.logits[0].clone()
        else:
            dec._step()
    assert torch.equal(dec.logits[0], replay)
    assert ops.ext().lib.lb_device_error() == 0


@torch.no_grad()
def test_greedy_continuation_is_the_argmax():
    """Free-running decode: each step's token is the argmax of that step's logits."""
    decode.enable_decode_options()
    dec = decode.Int4Decoder(decode.build(TINY, seed=5), max_len=48)
    dec.prefill(torch.arange(16) * 37 % TINY["vocab_size"])
    for _ in range(8):
        dec.step()
        assert dec.tok.item() == dec.logits[0].argmax().item()
    assert dec.pos.item() == 24
