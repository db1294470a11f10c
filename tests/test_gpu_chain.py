"""The device-resident code-predictor chain (src/families/qwen3-tts/talker.cpp:58-64, graph-sampler.cpp:20-64):
15 residual-codebook steps for 64 streams where each step's logits come from the previous step's drawn
ids (a GEMV of the gathered embedding rows) and nothing is read back between steps. The whole chain —
cuBLAS GEMVs standing in for the model, ssb_sample_embed_rows for the pick and the next get_rows — is
captured into one CUDA graph and replayed. Checked against the oracle on the logits each step actually
produced: ids identical (integers), statuses identical, and every gathered embedding row bit-identical
to the table row of its id."""
import numpy as np
import pytest

import speech_sampler as ss
from oracle import params as oparams

pytestmark = pytest.mark.gpu


def torch_mod():
    import torch
    return torch


def _build(torch, seed, B, H, V, G, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = torch.randn(G, H, V, device="cuda", generator=g) * (1.5 / H ** 0.5)
    E = torch.randn(G, V, H, device="cuda", generator=g).to(dtype)
    h0 = torch.randn(B, H, device="cuda", generator=g).to(dtype)
    u = torch.rand(G, B, device="cuda", generator=g, dtype=torch.float64)
    return W, E, h0, u


def _check(oracle, p, logits, ids, st, E, h, u):
    for step in range(logits.shape[0]):
        x = logits[step].cpu().numpy()
        op = oparams(greedy=bool(p.greedy), temperature=p.temperature, top_k=p.top_k, top_p=p.top_p)
        want, wst, _ = oracle.sample_rows(x, op, u=u[step].cpu().numpy())
        assert np.array_equal(st[step].cpu().numpy(), wst), step
        assert np.array_equal(ids[step].cpu().numpy(), want), step
        gathered = E[step][ids[step].long()]
        bits = {2: "int16", 4: "int32"}[gathered.element_size()]
        assert torch_mod().equal(h[step + 1].view(getattr(torch_mod(), bits)), gathered.view(getattr(torch_mod(), bits))), step


@pytest.mark.parametrize("greedy", [False, True])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_code_predictor_chain_in_a_cuda_graph(engine, oracle, greedy, dtype):
    torch = torch_mod()
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    B, H, V, G = 64, 256, 2048, 15
    W, E, h0, u = _build(torch, 5, B, H, V, G, tdt)
    p = ss.params(greedy=greedy, temperature=0.9, top_k=50, top_p=1.0)
    logits = torch.empty(G, B, V, device="cuda")
    ids = torch.empty(G, B, dtype=torch.int32, device="cuda")
    st = torch.empty(G, B, dtype=torch.int32, device="cuda")
    h = torch.empty(G + 1, B, H, device="cuda", dtype=tdt)
    uu = u.clone()

    def chain():
        for step in range(G):
            torch.matmul(h[step].float(), W[step], out=logits[step])
            engine.sample_embed(logits[step], p, E[step], h[step + 1], u=None if greedy else uu[step], ids=ids[step],
                                status=st[step], stream=torch.cuda.current_stream())

    side = torch.cuda.Stream()
    h[0].copy_(h0)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        chain()  # eager once (warm-up: kernel attributes, cuBLAS handles)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain()
    for trial in range(2):  # replay with fresh inputs copied into the graph's buffers
        g = torch.Generator(device="cuda").manual_seed(100 + trial)
        h[0].copy_(torch.randn(B, H, device="cuda", generator=g).to(tdt))
        uu.copy_(torch.rand(G, B, device="cuda", generator=g, dtype=torch.float64))
        graph.replay()
        torch.cuda.synchronize()
        _check(oracle, p, logits, ids, st, E, h, uu)


def test_refused_rows_gather_zeros(engine):
    torch = torch_mod()
    x = torch.randn(4, 2048, device="cuda")
    x[1, 7] = float("nan")
    table = torch.randn(2048, 96, device="cuda")
    out = torch.full((4, 100), 7.0, device="cuda")
    ids, st = engine.sample_embed(x, ss.params(greedy=True), table, out)
    torch.cuda.synchronize()
    assert st[1].item() == ss.ROW_NON_FINITE_INPUT and ids[1].item() == -1
    assert torch.all(out[1, :96] == 0) and torch.all(out[:, 96:] == 7.0)
    for r in (0, 2, 3):
        assert torch.equal(out[r, :96], table[ids[r].long()])
