"""The public ops can be captured in a CUDA graph: they launch on the
current stream, allocate nothing in the library, and the GLA sequence split
forks its library-owned side stream from, and joins it back to, the
capturing stream with events.  A replay must reproduce the eager result bit
for bit."""
import pytest
import torch

from glaucis_b200 import configs, ops

pytestmark = pytest.mark.gpu


def _capture(fn):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        fn()
    return graph


def test_gmm_forward_replays_bit_for_bit(cuda):
    cfg = configs.GMM_CONFIGS["gmm_small"]
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device=cuda, seed=1)
    a_q, a_s = ops.quant_act_1x128(lhs)
    b_q, b_s = ops.quant_w_128x128(rhs)
    out = torch.empty((cfg.M, cfg.N), dtype=torch.bfloat16, device=cuda)
    ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out=out)
    want = out.clone()
    graph = _capture(lambda: ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out=out))
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(out, want)


@pytest.mark.parametrize("B,T,H", [(2, 512, 16), (1, 4096, 4)])
def test_gla_forward_replays_bit_for_bit(cuda, B, T, H):
    # (1, 4096, 4) takes the sequence split: state-only pass on the side
    # stream beside segment 0, the fold, then the other segments
    cfg = configs.GLAConfig("t", B=B, T=T, H=H, h0_std=0.1)
    inp = configs.make_gla_inputs(cfg, device=cuda, seed=4)
    o = torch.empty_like(inp["v"])
    ht = torch.empty_like(inp["h0"])

    def fn():
        ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], None, 128 ** -0.5, 64, g=inp["g"],
                          h0=inp["h0"], output_final_state=True, o=o, ht=ht)

    fn()
    want_o, want_ht = o.clone(), ht.clone()
    graph = _capture(fn)
    o.zero_()
    ht.zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    assert torch.equal(o, want_o) and torch.equal(ht, want_ht)
