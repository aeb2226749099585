"""GPU parity of the chained decode step: several BASELINE config-5 layers (paged GQA
attention B=32 x 4096, Hq=32, Hkv=8 -> W8A16 SwiGLU MoE E=8 top-2, d=4096, F=14336, T=32)
captured in ONE CUDA graph, each layer with its own KV cache and experts, the attention
output [32, 4096] feeding the MoE and the MoE output becoming the next layer's q (the
reference's graph-captured multi-layer decode step, 03_moe_wq_decode.cu:651-681).

Every layer is checked against the fp64 oracle on the input the GPU actually gave it:
attention on sampled sequences (out max-abs <= 2e-3, lse <= 1e-4 abs + 1e-4 rel,
01_decode_attention.cu:776), the MoE block's routing ids bit-exact for all 32 tokens and
its output on 8 sampled tokens (rel-RMS <= 1e-2).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HQ, HKV, D, PAGE = 32, 8, 128, 16
OUT_ATOL = 2e-3
LSE_ATOL, LSE_RTOL = 1e-4, 1e-4
REL_RMS = 1e-2


def _layer(ckl, oracle, dev, B, L, E, d, F, seed):
    import torch
    bt = oracle.batch([L] * B, HQ, HKV, seed, fill=False)      # shuffled page table
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    shape = (bt.num_pages, PAGE, HKV, D)
    kc = (torch.rand(shape, generator=g, device=dev) * 2 - 1).half()
    vc = (torch.rand(shape, generator=g, device=dev) * 2 - 1).half()
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    attn = dict(k_cache=kc, v_cache=vc, kv_indptr=t(bt.indptr), kv_indices=t(bt.indices),
                kv_last_page_len=t(bt.last))
    nc, ct = ckl.plan_chunks(HQ // HKV, B, HKV, L)
    mk = lambda *sh: (torch.randn(*sh, generator=g, device=dev) * 0.02).half()
    q = [ckl.QuantWeights(8, mk(E, d, F), group=d), ckl.QuantWeights(8, mk(E, d, F), group=d),
         ckl.QuantWeights(8, mk(E, F, d), group=F)]
    k = 2
    return dict(bt=bt, attn=attn, nc=nc, ct=ct, q=q, moe=ckl.MoeLayer(*q),
                lg=torch.randn((B, E), generator=g, device=dev),
                a_out=torch.empty((B, HQ, D), dtype=torch.float16, device=dev),
                a_lse=torch.empty((B, HQ), dtype=torch.float32, device=dev),
                a_ws=torch.empty(1 << 24, dtype=torch.uint8, device=dev),
                h=torch.empty((B, d), dtype=torch.float16, device=dev),
                ids=torch.empty((B, k), dtype=torch.int32, device=dev),
                m_ws=None)


def _check_attention(oracle, ly, q_in, seqs):
    """The layer's attention rows of `seqs` against the fp64 oracle, from q_in (host)."""
    import torch
    bt, kc, vc = ly["bt"], ly["attn"]["k_cache"], ly["attn"]["v_cache"]
    out = ly["a_out"].float().cpu().numpy()
    lse = ly["a_lse"].cpu().numpy()
    for b in seqs:
        pages = bt.indices[bt.indptr[b]:bt.indptr[b + 1]]
        pi = torch.from_numpy(pages.astype(np.int64)).to(kc.device)
        sb = oracle.Batch([bt.lens[b]], HQ, HKV, np.array([0, len(pages)], np.int32),
                          np.arange(len(pages), dtype=np.int32), bt.last[b:b + 1],
                          np.ascontiguousarray(q_in[b:b + 1]), kc.index_select(0, pi).cpu().numpy(),
                          vc.index_select(0, pi).cpu().numpy())
        ro, rl = oracle.attention_ref(sb)
        err = np.abs(out[b] - ro[0]).max()
        assert err <= OUT_ATOL, f"seq {b}: attention out max-abs {err:.3e}"
        assert np.all(np.abs(lse[b] - rl[0]) <= LSE_ATOL + LSE_RTOL * np.abs(rl[0])), f"seq {b}: lse"


@pytest.mark.parametrize("n_layers", [2])
def test_chained_config5_step_in_one_graph(ckl, oracle, dev, n_layers):
    import torch
    from moe_ref import rel_rms, sample_tokens, sampled_layer_ref
    B, L, E, k, d, F = 32, 4096, 8, 2, 4096, 14336
    layers = [_layer(ckl, oracle, dev, B, L, E, d, F, seed=300 + l) for l in range(n_layers)]
    m_ws = torch.empty(layers[0]["moe"].workspace_size(B, k), dtype=torch.uint8, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(299)
    q0 = (torch.rand((B, HQ, D), generator=g, device=dev) * 2 - 1).half()

    def step():
        x = q0
        for ly in layers:
            ckl.decode_attention(x.view(B, HQ, D), **ly["attn"], num_chunks=ly["nc"],
                                 chunk_tokens=ly["ct"], out=ly["a_out"], lse=ly["a_lse"],
                                 workspace=ly["a_ws"])
            ly["moe"].forward(ly["lg"], ly["a_out"].view(B, d), k, out=ly["h"], ids=ly["ids"],
                              workspace=m_ws)
            x = ly["h"]

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()                                         # first calls outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for ly in layers:                                  # the replay must rewrite every output
        for key in ("a_out", "h"):
            ly[key].fill_(float("nan"))
        ly["ids"].fill_(-1)
    graph.replay()
    torch.cuda.synchronize()
    ckl.check_device_error()

    q_in = q0.cpu().numpy()
    for l, ly in enumerate(layers):
        _check_attention(oracle, ly, q_in, seqs=(0, 13, B - 1))
        x = ly["a_out"].view(B, d).cpu().numpy()
        tok = sample_tokens(B)
        ref, rids = sampled_layer_ref(oracle, ly["lg"].cpu().numpy(), x, k, *ly["q"], tok)
        assert np.array_equal(ly["ids"].cpu().numpy(), rids), f"layer {l}: routing ids"
        rr = rel_rms(ly["h"].float().cpu().numpy()[tok], ref)
        assert rr <= REL_RMS, f"layer {l}: MoE rel-RMS {rr:.3e}"
        q_in = ly["h"].view(B, HQ, D).cpu().numpy()

    # a second replay gives the same bits (the step is deterministic)
    first = [ly["h"].clone() for ly in layers]
    graph.replay()
    torch.cuda.synchronize()
    for a, ly in zip(first, layers):
        assert torch.equal(a, ly["h"])
    del graph, layers
    torch.cuda.empty_cache()
