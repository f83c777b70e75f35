"""Data parallelism on two GPUs (skipped on a one-GPU box): two NCCL ranks, each its own micro-batch through
the same base and adapter, the step captured as one CUDA graph with the gradient exchange captured in it
(dp.GradBuckets inside model.GraphStep): per-layer all-reduces on a side stream, or one all-reduce after the
backward (the bench's default).

Checked: the gradient each rank holds after a captured step with the exchange equals the mean of the two
ranks' own eager gradients (exchanged with a plain all-gather), and after steps with AdamW inside the graph
the two ranks' adapters are bit-identical. Each rank runs as a spawned child process with a short process
group timeout; NVLS is off (NCCL_NVLS_ENABLE=0)."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out, overlap):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                           timeout=datetime.timedelta(seconds=120))
    graph = None
    try:
        from r97training_b200.dp import GradBuckets
        from r97training_b200.model import Adapter, GraphStep, HybridConfig, HybridModel, TrainStep
        cfg = HybridConfig(hidden=256, layers=4, gdn_heads=4, gdn_qk_heads=2, attn_heads=2, attn_kv_heads=1,
                           ffn=512, vocab=1024, rank=8, alpha=16.0, seq=128, micro_batch=2, lr=1e-3)
        model = HybridModel(cfg, dev)
        ad = Adapter(model, dev, b_std=2e-2)
        step = TrainStep(model, ad, head_chunk=128)
        gen = torch.Generator(device=dev)
        gen.manual_seed(100 + rank)
        ids = [torch.randint(0, cfg.vocab, (cfg.micro_batch, cfg.seq), device=dev, generator=gen,
                             dtype=torch.int32) for _ in range(3)]
        # this rank's own gradient, eagerly, no exchange; the mean of both ranks' by an all-gather
        step.run(ids[0])
        own = ad.g.clone()
        both = [torch.empty_like(own) for _ in range(world)]
        dist.all_gather(both, own)
        mean = sum(both) / world
        ad.g.zero_()
        # the eager exchange once (collectives and buffers set up outside any capture)
        buckets = GradBuckets(ad.g, ad.layer_ranges, overlap=overlap)
        step.grad_hook = buckets.ready
        step.run(ids[0])
        buckets.join()
        ad.g.zero_()
        torch.cuda.synchronize()
        graph = GraphStep(step, ids[0], update=False, buckets=buckets)
        graph.replay(ids[0])
        torch.cuda.synchronize()
        rel = float((ad.g - mean).norm() / mean.norm())
        graph.release()
        graph = None
        # steps with the update inside the graph: the ranks' adapters stay identical
        ad.g.zero_()
        graph = GraphStep(step, ids[1], update=True, buckets=buckets)
        for b in ids[1:]:
            graph.replay(b)
        torch.cuda.synchronize()
        w = ad.w.clone()
        ws = [torch.empty_like(w) for _ in range(world)]
        dist.all_gather(ws, w)
        same = all(torch.equal(ws[0], x) for x in ws[1:])
        out[rank] = (rel, same, int(ad.step))
    finally:
        if graph is not None:
            graph.release()
        dist.destroy_process_group()


@pytest.mark.parametrize("overlap", [True, False])
def test_two_rank_captured_exchange(overlap):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, out, overlap)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(600)
        for p in procs:
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(out)
    for r in range(2):
        rel, same, steps = res[r]
        assert rel <= 1e-4, (r, rel)
        assert same, r
        assert steps == 2, steps
