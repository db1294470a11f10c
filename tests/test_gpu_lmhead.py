"""The LM head fused with its argmax (ssb_lm_head_argmax: tcgen05 MMAs, argmax in the TMEM epilogue,
Qwen3Readback::Pick / verify, src/common/qwen3-decoder.cpp:422-437, 492-510) against a plain PyTorch fp32
reference of the same op: logits = hidden.float() @ weight.float().T, first argmax.

Tolerance: both sides accumulate the same bf16 products in fp32, in different orders, so a logit may
differ by about dim x 2^-24 x sum |products|; the test allows 1e-3 (absolute, logits of magnitude ~5).
The id must equal torch's first argmax wherever the two best logits of torch are farther apart than
that; otherwise the engine's logit must lie within it of torch's maximum. max_logit within the same."""
import pytest

import speech_sampler as ss

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.mark.parametrize("rows,dim,vocab", [(1, 1024, 151936), (3, 2048, 151936), (16, 1024, 32000),
                                            (64, 2048, 151936), (256, 1024, 151936), (5, 64, 1000),
                                            (17, 128, 129), (40, 192, 3000)])
def test_lm_head_argmax_matches_torch(engine, rows, dim, vocab):
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    g = torch.Generator(device="cuda").manual_seed(rows * 1000 + dim)
    hidden = torch.randn(rows, dim, device="cuda", generator=g).to(torch.bfloat16)
    weight = (torch.randn(vocab, dim, device="cuda", generator=g) * (2.0 / dim ** 0.5)).to(torch.bfloat16)
    ids = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    mx = torch.empty(rows, device="cuda")
    st = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    for call in range(2):  # the second call checks that the first left the context's maxima cleared
        engine.lm_head_argmax(hidden, weight, ids, mx, st)
        torch.cuda.synchronize()
        logits = hidden.float() @ weight.float().T
        want = torch.argmax(logits, dim=1)
        top2 = torch.topk(logits, 2, dim=1).values
        assert torch.all(st == ss.ROW_OK)
        for r in range(rows):
            got = int(ids[r])
            assert 0 <= got < vocab
            if float(top2[r, 0] - top2[r, 1]) > TOL:
                assert got == int(want[r]), (call, r, got, int(want[r]))
            else:
                assert float(top2[r, 0] - logits[r, got]) <= TOL
            assert abs(float(mx[r]) - float(top2[r, 0])) <= TOL


def test_lm_head_ties_take_the_lowest_token(engine):
    import torch
    dim, vocab = 128, 4096
    hidden = torch.zeros(2, dim, device="cuda", dtype=torch.bfloat16)
    hidden[:, 0] = 1.0
    weight = torch.zeros(vocab, dim, device="cuda", dtype=torch.bfloat16)
    weight[[77, 300, 4000], 0] = 2.0  # three equal maxima, in three tiles
    weight[5, 0] = -1.0
    ids = engine.lm_head_argmax(hidden, weight)
    torch.cuda.synchronize()
    assert ids.tolist() == [77, 77]
    weight.zero_()  # every logit 0: the first token
    ids = engine.lm_head_argmax(hidden, weight)
    torch.cuda.synchronize()
    assert ids.tolist() == [0, 0]


def test_lm_head_refusals(engine):
    import torch
    h = torch.zeros(2, 100, device="cuda", dtype=torch.bfloat16)  # dim not a multiple of 64
    w = torch.zeros(50, 100, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ss.SsbError):
        engine.lm_head_argmax(h, w)
    h = torch.zeros(300, 64, device="cuda", dtype=torch.bfloat16)  # more than 256 rows
    w = torch.zeros(50, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ss.SsbError) as e:
        engine.lm_head_argmax(h, w)
    assert e.value.status == ss.OUT_OF_RANGE
