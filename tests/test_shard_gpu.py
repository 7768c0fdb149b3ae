"""The expert-sharded grouped matmul whose epilogue writes every rank's
output buffer (shard.gmm_fp8_fwd_gathered over shard.PeerBuffers), run as a
one-rank NCCL group on one GPU: the rank's rows go through the TMA-store
scatter epilogue into its IPC-allocated buffer at the shard's row offset and
must equal the plain one-GPU matmul bit for bit.  (With several GPUs the
same call also stores into the peers' buffers; bench.py measures that.)"""
import pytest
import torch

from glaucis_b200 import configs, ops, shard

pytestmark = pytest.mark.gpu


@pytest.fixture
def one_rank_group(cuda):
    import torch.distributed as dist
    if dist.is_initialized():
        pytest.skip("a process group already exists")
    import socket
    with socket.socket() as sk:  # a free local port for the one-rank rendezvous
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            device_id=torch.device(cuda))
    yield
    dist.destroy_process_group()


def test_gathered_matmul_equals_one_gpu(cuda, one_rank_group):
    cfg = configs.GMMConfig("t", G=6, M=1536, K=1024, N=512, routing="uniform_one_empty")
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device=cuda, seed=31)
    a_q, a_s = ops.quant_act_1x128(lhs)
    b_q, b_s = ops.quant_w_128x128(rhs)
    want = ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out_dtype=torch.bfloat16)
    (me,) = shard.gmm_partition(gs.cpu().numpy(), 1)
    peers = shard.PeerBuffers(me.rows, cfg.N)
    try:
        peers.local.fill_(7.0)
        got = shard.gmm_fp8_fwd_gathered(a_q[me.r0:me.r1], a_s[me.r0:me.r1], b_q[me.g0:me.g1],
                                         b_s[me.g0:me.g1], me, peers)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        rows = int(gs.sum().item())
        assert torch.equal(got[:rows], want[:rows])
    finally:
        peers.close()


def test_gathered_matmul_two_calls_with_different_inputs(cuda, one_rank_group):
    # The result is the shared buffer itself: the second call overwrites it, so
    # the first result is cloned before that call; both must equal one GPU.
    cfg = configs.GMMConfig("t2", G=4, M=1024, K=512, N=256, routing="uniform_one_empty")
    (me,) = shard.gmm_partition(configs.group_sizes(cfg.routing, cfg.G, cfg.M, seed=41), 1)
    peers = shard.PeerBuffers(cfg.M, cfg.N)
    try:
        outs, wants = [], []
        for seed in (41, 42):
            lhs, rhs, _ = configs.make_gmm_inputs(cfg, device=cuda, seed=seed)
            gs = torch.from_numpy(me.sizes).to(cuda)
            a_q, a_s = ops.quant_act_1x128(lhs)
            b_q, b_s = ops.quant_w_128x128(rhs[me.g0:me.g1].contiguous())
            wants.append(ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out_dtype=torch.bfloat16))
            outs.append(shard.gmm_fp8_fwd_gathered(a_q, a_s, b_q, b_s, me, peers, gs).clone())
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        assert not torch.equal(wants[0], wants[1])
        for got, want in zip(outs, wants):
            assert torch.equal(got, want)
    finally:
        peers.close()


@pytest.mark.parametrize("B,T,H", [(1, 2048, 4), (2, 512, 80)])
def test_gathered_gla_equals_one_gpu(cuda, one_rank_group, B, T, H):
    # The head-sharded GLA forward whose kernel stores O into block `rank` of
    # every rank's buffer (one rank: its own block).  (1, 2048, 4) runs the
    # sequence split (O from both full passes), (2, 512, 80) one CTA per
    # (batch, head).  Both equal the plain forward bit for bit.
    cfg = configs.GLAConfig("t", B=B, T=T, H=H, h0_std=0.1)
    inp = configs.make_gla_inputs(cfg, device=cuda, seed=33)
    want = ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], None, 128 ** -0.5, 64, g=inp["g"],
                             h0=inp["h0"], output_final_state=True)
    width = B * T * H * 128 + 256  # a padded block, like unequal head counts need
    peers = shard.PeerBuffers(1, width)
    try:
        peers.local.fill_(7.0)
        ht = torch.empty_like(inp["h0"])
        got = shard.gla_fwd_gathered(inp["q"], inp["k"], inp["v"], inp["g"], inp["h0"],
                                     128 ** -0.5, peers, width, ht=ht)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        blk = got[0, : B * T * H * 128].view(B, T, H, 128)
        assert torch.equal(blk, want.o)
        assert torch.equal(ht, want.ht)
        assert torch.all(got[0, B * T * H * 128:] == 7.0)  # the padding is not written
    finally:
        peers.close()


@pytest.mark.parametrize("B,T,H", [(2, 256, 80), (1, 2048, 4)])
def test_gla_scatter_writes_every_output(cuda, B, T, H):
    # the raw op with three local outputs (the scatter instance), both
    # precisions; (1, 2048, 4) takes the sequence split, whose two full
    # passes both store O
    cfg = configs.GLAConfig("t", B=B, T=T, H=H)
    inp = configs.make_gla_inputs(cfg, device=cuda, seed=34)
    for exact in (True, False):
        want = ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], None, 128 ** -0.5, 64, g=inp["g"],
                                 exact_intra=exact).o
        outs = [torch.full_like(want, 3.0) for _ in range(3)]
        ops.chunk_gla_fwd_scatter(inp["q"], inp["k"], inp["v"], None, 128 ** -0.5, 64, outs=outs,
                                  g=inp["g"], exact_intra=exact)
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        for o in outs:
            assert torch.equal(o, want)
