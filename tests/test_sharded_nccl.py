"""Column-sharded layers over NCCL on 2 GPUs (skipped with fewer GPUs).

Each rank runs the B200 kernels on its shard; the all-gathered output must
match the CPU oracle of the full layer, eagerly and replayed from a CUDA
graph that contains the kernel and the NCCL collective.  The all-gather over
NVLink peer memory (PeerGather) must give the same bits as NCCL's, over
consecutive calls with changing inputs and from graph replays.
"""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import qlinear_oracle as orc

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, result_q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        from qlinear.quantization.int4 import QuantizedLinearInt4
        from qlinear.quantization.int8 import QuantizedLinearInt8
        from qlinear.sharded import ShardedQuantizedLinear
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        K, N, M, wbits, groups = case
        g = torch.Generator().manual_seed(5)
        lin = torch.nn.Linear(K, N, bias=False).half()
        with torch.no_grad():
            lin.weight.copy_((torch.randn(N, K, generator=g) * 0.02).half())
        q = QuantizedLinearInt4.from_linear(lin) if wbits == 4 else QuantizedLinearInt8.from_linear(lin)
        x = torch.randn(M, K, generator=g).half()
        sh = ShardedQuantizedLinear.from_quantized(q, rank, world, groups=groups).cuda()
        xd = x.cuda()
        y = sh(xd)
        # graph replay of the sharded forward (kernel + NCCL all-gather)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            sh(xd)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                yg = sh(xd)
        torch.cuda.current_stream().wait_stream(s)
        graph.replay()
        torch.cuda.synchronize()
        if wbits == 4:
            deq = orc.dequantize_int4(q.weight_packed.numpy(), q.scales.numpy())
        else:
            deq = orc.dequantize_int8(q.weight_q.numpy(), q.scale.numpy())
        ref = orc.linear_f32(x.numpy(), deq)
        ok, max_abs, rel, b_abs, b_rel = orc.check_parity(y.float().cpu().numpy(), ref, x.numpy(), deq)
        same = torch.equal(y, yg)
        if groups == 1:   # sharded argmax: keys all-gathered, equals argmax of the gathered logits
            want = torch.argmax(y, dim=-1)
            same = same and torch.equal(sh.argmax(xd), want)
            # the same through the NVLink exchange kernel, eager and from a graph;
            # up to 8 rows the shard's linear runs unsplit with the exchange in its
            # epilogue, so its expectation is the argmax of the unsplit outputs
            from helpers import linear_unsplit
            from qlinear.p2p import PeerExchange
            if M <= 8:
                ref_sh = ShardedQuantizedLinear(sh.local, sh.out_features, rank, world, local_fn=linear_unsplit)
                want = torch.argmax(ref_sh(xd), dim=-1)
            sh.exchange = PeerExchange(rank, world, max_m=64)
            same = same and torch.equal(sh.argmax(xd), want)
            with torch.cuda.stream(s):
                g2 = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g2, stream=s):
                    ig = sh.argmax(xd)
            torch.cuda.current_stream().wait_stream(s)
            for _ in range(4):
                ig.zero_()
                g2.replay()
                torch.cuda.synchronize()
                same = same and torch.equal(ig, want)
            del g2
            sh.exchange.close()
            from qlinear import _lib
            same = same and _lib.device_error() == 0
        # the all-gather over peer memory: same bits as NCCL's, call after
        # call (the two banks alternate) and from graph replays
        from qlinear.p2p import PeerGather
        xs = [torch.randn(M, K, generator=g).half().cuda() for _ in range(3)]
        want = [sh(xi) for xi in xs]
        sh.gatherer = PeerGather(rank, world, max_m=64, n_cols=N)
        for i in range(5):
            same = same and torch.equal(sh(xs[i % 3]), want[i % 3])
        xstat = xs[0].clone()
        with torch.cuda.stream(s):
            sh(xstat)
            torch.cuda.synchronize()
            g3 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g3, stream=s):
                yp = sh(xstat)
        torch.cuda.current_stream().wait_stream(s)
        for i in range(5):
            xstat.copy_(xs[(i + 1) % 3])
            g3.replay()
            torch.cuda.synchronize()
            same = same and torch.equal(yp, want[(i + 1) % 3])
        del g3
        sh.gatherer.close()
        sh.gatherer = None
        from qlinear import _lib
        same = same and _lib.device_error() == 0
        del graph
        dist.barrier()
        dist.destroy_process_group()
        result_q.put((rank, bool(ok and same), max_abs, rel))
    except Exception as e:
        result_q.put((rank, False, repr(e)[:300], None))


# the peer all-gather sends the first case through its flagged banks 2 bytes
# at a time (odd widths), the last one with 16-byte stores (5 MB of output),
# the others as tagged lines
@pytest.mark.parametrize("case", [(1536, 8192 + 37, 1, 4, 1), (4096, 2 * 1792, 16, 8, 2), (1536, 4096, 64, 4, 1),
                                  (4096, 16032 * 2, 3, 8, 1), (1536, 40960, 64, 4, 1)])
def test_sharded_nccl_two_gpus(case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = sorted(q.get() for _ in range(q.qsize()) if True) if not q.empty() else []
    assert len(res) == 2, (res, [p.exitcode for p in procs])
    for rank, ok, a, b in res:
        assert ok, (rank, a, b)


def _gather_worker(rank, world, port, result_q):
    """Back-to-back flagged all-gathers (5 MB of output each, over the 4 MB
    tagged-line limit) with no host synchronisation between the calls: a
    fast rank may already have published call e + 1 while a slow one still
    waits for call e, which the wait must accept."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        from qlinear import _lib
        from qlinear.p2p import PeerGather
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        M, N, calls = 64, 40960, 8
        block = (N + world - 1) // world
        lo, hi = rank * block, min(N, (rank + 1) * block)
        gat = PeerGather(rank, world, max_m=M, n_cols=N)
        outs = [torch.zeros(M, N, dtype=torch.float16, device="cuda") for _ in range(calls)]
        dist.barrier()
        for c, o in enumerate(outs):
            o[:, lo:hi] = float(rank * 16 + c)
            gat.gather(o, block)
        torch.cuda.synchronize()
        ok = _lib.device_error() == 0
        for c, o in enumerate(outs):
            want = torch.empty(M, N, dtype=torch.float16, device="cuda")
            for q in range(world):
                want[:, q * block:min(N, (q + 1) * block)] = float(q * 16 + c)
            ok = ok and torch.equal(o, want)
        gat.close()
        dist.barrier()
        dist.destroy_process_group()
        result_q.put((rank, bool(ok), None, None))
    except Exception as e:
        result_q.put((rank, False, repr(e)[:300], None))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_gather_back_to_back_flagged(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = sorted(q.get() for _ in range(q.qsize())) if not q.empty() else []
    assert len(res) == world, (res, [p.exitcode for p in procs])
    for rank, ok, a, b in res:
        assert ok, (rank, a, b)
