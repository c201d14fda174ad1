"""Peer-memory data parallelism on B200: the bounded wait, the reduce-scatter
kernel against a torch sum, and the trainer against FSDP2 (2 GPUs)."""
import os
import socket
import tempfile

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def test_dp_barrier_gives_up_and_reports():
    """A wait on a flag that nothing sets ends after its limit with an error code;
    the context stays usable."""
    from torchtitan_b200.ops._ext import ext

    from torchtitan_b200.parallel.watchdog import install

    e = ext()
    e.dp_error_code(True)
    wd = install(e)
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    # world 2 with both "peers" pointing at this GPU's flags: slot entry of rank 1 is never written
    e.dp_barrier([flags.data_ptr(), flags.data_ptr()], 0, 1, 1, limit_s=0.2)
    torch.cuda.synchronize()
    assert e.dp_error_code(True) == 72
    assert int(flags[2]) == 1 and int(flags[3]) == 0
    # the pinned host word saw it too: slot 1, epoch 1, source rank 1, flag value 0
    assert wd.poll() is not None and wd.error[:5] == [72, 1, 1, 1, 0]
    wd.reset()
    assert float(torch.ones(4, device="cuda").sum()) == 4.0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _entry(rank, world, port, fn, args):
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world), LOCAL_WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        fn(rank, world, *args)
    finally:
        dist.destroy_process_group()


def _run(fn, world, *args):
    mp.spawn(_entry, args=(world, _port(), fn, args), nprocs=world, join=True)


two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


def _rs(rank, world):
    from torch.distributed.device_mesh import init_device_mesh

    from torchtitan_b200.parallel.peer_dp import PeerDataParallel

    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(1000, 3000), torch.nn.Linear(3000, 515)).cuda()
    mesh = init_device_mesh("cuda", (world,))
    rt = PeerDataParallel(model, mesh, bucket_mb=2)
    assert len(rt.buckets) >= 2
    rt.begin_microbatch(0, 1)
    g = torch.Generator(device="cuda").manual_seed(1 + rank)
    x = torch.randn(64, 1000, device="cuda", dtype=torch.bfloat16, generator=g)
    model(x).float().square().mean().backward()
    rt.finish_backward()
    torch.cuda.synchronize()
    assert rt._ext.dp_error_code(True) == 0
    # reference: every rank's bf16 gradient buffer summed in fp32, this rank's slices
    full = rt.gbuf.float().clone()
    dist.all_reduce(full)
    for b, shard in zip(rt.buckets, rt.shard_views(rt.grad_shard)):
        sl = b.shard_len(world)
        torch.testing.assert_close(shard, full[b.offset + rank * sl:b.offset + (rank + 1) * sl], rtol=1e-5,
                                   atol=1e-6)
    # optimizer: fp32 masters updated, new bf16 weights written into every rank's buffer
    m, v = torch.zeros_like(rt.master), torch.zeros_like(rt.master)
    before = rt.wbuf.clone()
    rt.adamw_step(m, v, lr=1e-2, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, step=1, clip=None)
    torch.cuda.synchronize()
    assert rt._ext.dp_error_code(True) == 0
    ws = [torch.empty_like(rt.wbuf) for _ in range(world)]
    dist.all_gather(ws, rt.wbuf)
    assert torch.equal(ws[0], ws[1]) and not torch.equal(rt.wbuf, before)
    for b, shard in zip(rt.buckets, rt.shard_views(rt.master)):
        sl = b.shard_len(world)
        assert torch.equal(rt.wbuf[b.offset + rank * sl:b.offset + (rank + 1) * sl], shard.bfloat16())


@two_gpus
def test_peer_reduce_scatter_and_fused_all_gather():
    _run(_rs, 2)


def _trainer(rank, world, out_dir):
    from torch.distributed.checkpoint.state_dict import StateDictOptions, get_model_state_dict

    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    def make(comm):
        return Trainer(ConfigManager().parse_args([
            "--module", "llama3", "--config", "llama3_debugmodel", "--training.steps", "6",
            "--metrics.log-freq", "1", "--parallelism.data-parallel-comm", comm, "--dump-folder",
            os.path.join(out_dir, comm), "--training.global-batch-size", "16"]))

    tf, tp = make("fsdp2"), make("peer")
    assert getattr(tf.model_parts[0], "_dp_runtime", None) is None
    assert tp.model_parts[0]._dp_runtime.comm == "peer"
    full = get_model_state_dict(tf.model_parts[0], options=StateDictOptions(full_state_dict=True))
    tp.checkpointer.states["model"].load_state_dict(full)  # same starting weights
    res = {}
    for name, t in (("fsdp2", tf), ("peer", tp)):
        t.train()
        m = t.metrics_processor.last_metrics
        res[name] = (m["loss_metrics/global_avg_loss"], m["grad_norm"])
    # bf16 compute on both sides: FSDP2 reduces in fp32, the peer kernel sums bf16 grads in fp32
    assert abs(res["peer"][0] - res["fsdp2"][0]) < 2e-2, res
    assert abs(res["peer"][1] - res["fsdp2"][1]) < 5e-2 * res["fsdp2"][1], res
    tp.model_parts[0]._dp_runtime.check()
    tf.close()
    tp.close()


@two_gpus
def test_peer_data_parallel_trainer_two_gpus():
    with tempfile.TemporaryDirectory() as d:
        _run(_trainer, 2, d)


def _ep_peer(rank, world):
    from torchtitan_b200.models.common.moe import MoE
    from torchtitan_b200.parallel.ep_fused import make_fused_ep_dispatch

    torch.manual_seed(0)
    E = 4 * world
    m = MoE(256, 512, num_experts=E, top_k=2, load_balance_coeff=None).cuda()
    m.init_weights(0.05)
    for p in m.parameters():
        dist.broadcast(p.data, 0)
    m = m.to(torch.bfloat16)
    x = torch.randn(1, 300 + 64 * rank, 256, device="cuda", dtype=torch.bfloat16,
                    generator=torch.Generator(device="cuda").manual_seed(rank)).requires_grad_()
    ref = m(x)
    ref.float().square().sum().backward()
    gx_ref = x.grad.clone()
    e = m.experts
    for name in ("w1", "w2", "w3"):
        setattr(e, name, torch.nn.Parameter(getattr(e, name).data[rank * 4:(rank + 1) * 4].clone()))
    m.ep_dispatch = make_fused_ep_dispatch(dist.group.WORLD, E)
    for _ in range(2):  # the second call queues its row stores before the host sees the counts
        xr = x.detach().clone().requires_grad_()
        out = m(xr)
        assert m.ep_dispatch.comm.comm == "peer"
        torch.testing.assert_close(out.float(), ref.float(), rtol=2e-2, atol=2e-2)
        out.float().square().sum().backward()
        torch.testing.assert_close(xr.grad.float(), gx_ref.float(), rtol=5e-2, atol=5e-2)
    torch.cuda.synchronize()
    from torchtitan_b200.ops._ext import ext

    assert ext().dp_error_code(True) == 0
    assert ext().ep_error_code(True) == 0  # no peer row index fell outside its buffer


@two_gpus
def test_fused_expert_parallel_peer_memory():
    _run(_ep_peer, 2)
