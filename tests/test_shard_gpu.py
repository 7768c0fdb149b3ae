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
