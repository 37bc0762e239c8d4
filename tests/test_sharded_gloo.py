"""Column-sharded layers (qlinear.sharded) on CPU ranks over gloo.

The sharding, padding, all-gather and reassembly logic is the same code
that runs over NCCL on GPUs; here each rank's local compute is the CPU
oracle, and the gathered result must equal the oracle on the full layer.
A rank that dies before the collective must make the other rank fail
(within the process-group timeout), not hang.
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


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_local(module, x2):
    from qlinear.quantization.int4 import QuantizedLinearInt4
    if isinstance(module, QuantizedLinearInt4):
        deq = orc.dequantize_int4(module.weight_packed.numpy(), module.scales.numpy(), module.layout)
    else:
        deq = orc.dequantize_int8(module.weight_q.numpy(), module.scale.numpy())
    b = module.bias.numpy() if module.bias is not None else None
    return torch.from_numpy(orc.linear_f32(x2.numpy(), deq, b).astype(np.float16))


def _cpu_keys(y, col_offset):
    """Checker restatement of the argmax key (value order, then smallest column)."""
    bits = y.contiguous().view(torch.int16).to(torch.int64) & 0xFFFF
    bits = torch.where(bits == 0x8000, torch.zeros_like(bits), bits)
    bits = torch.where((bits & 0x7FFF) > 0x7C00, torch.full_like(bits, 0x7FFF), bits)
    ordv = torch.where(bits >= 0x8000, 0xFFFF - bits, bits | 0x8000)
    cols = torch.arange(y.shape[1], dtype=torch.int64) + col_offset
    return ((ordv << 32) | (0xFFFFFFFF - cols)).amax(dim=1)


def _full_layer(K, N, wbits, seed):
    from qlinear.quantization.int4 import QuantizedLinearInt4
    from qlinear.quantization.int8 import QuantizedLinearInt8
    g = torch.Generator().manual_seed(seed)
    lin = torch.nn.Linear(K, N, bias=True).half()
    with torch.no_grad():
        lin.weight.copy_((torch.randn(N, K, generator=g) * 0.02).half())
        lin.bias.copy_((torch.randn(N, generator=g) * 0.1).half())
    q = QuantizedLinearInt4.from_linear(lin) if wbits == 4 else QuantizedLinearInt8.from_linear(lin)
    return lin, q


def _worker(rank, world, port, case, result_q):
    import sys
    from qlinear.sharded import ShardedQuantizedLinear
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=20))
        K, N, M, wbits, groups, mode = case
        lin, q = _full_layer(K, N, wbits, seed=7)
        if mode == "tie":
            # columns 5 and N-3 hold the same weights and the largest bias: the
            # argmax is the smaller column on every row
            from qlinear.quantization.int4 import QuantizedLinearInt4
            from qlinear.quantization.int8 import QuantizedLinearInt8
            with torch.no_grad():
                lin.weight[N - 3].copy_(lin.weight[5])
                lin.bias[5] = lin.bias[N - 3] = 30.0
            q = QuantizedLinearInt4.from_linear(lin) if wbits == 4 else QuantizedLinearInt8.from_linear(lin)
        if mode == "from_linear":
            sh = ShardedQuantizedLinear.from_linear(lin, wbits, rank, world, groups=groups, local_fn=_oracle_local)
        else:
            sh = ShardedQuantizedLinear.from_quantized(q, rank, world, groups=groups, local_fn=_oracle_local,
                                                       key_fn=_cpu_keys)
        g = torch.Generator().manual_seed(11)
        x = torch.randn(M, K, generator=g).half()
        if mode == "die" and rank == 1:
            os._exit(3)                                   # leaves before the collective
        if mode in ("argmax", "tie"):
            idx = sh.argmax(x)
            want = torch.argmax(_oracle_local(q, x), dim=-1)
            ok = torch.equal(idx, want) and (mode != "tie" or bool((idx == 5).all()))
            result_q.put((rank, "ok" if ok else "mismatch", f"{idx.tolist()} vs {want.tolist()}"))
            dist.destroy_process_group()
            return
        try:
            y = sh(x)
        except Exception as e:                            # the surviving rank must see an error
            result_q.put((rank, "error", type(e).__name__))
            return
        y_full = _oracle_local(q, x)
        ok = torch.equal(y, y_full)
        result_q.put((rank, "ok" if ok else "mismatch", float((y.float() - y_full.float()).abs().max())))
        dist.destroy_process_group()
    except Exception as e:
        result_q.put((rank, "exception", repr(e)[:200]))


def _run(world, case, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
    res = []
    while not q.empty():
        res.append(q.get())
    return sorted(res), [p.exitcode for p in procs]


@pytest.mark.parametrize("world,case", [
    (2, (256, 301, 3, 4, 1, "from_quantized")),     # uneven shards (151 + 150), int4
    (2, (128, 260, 2, 8, 2, "from_quantized")),     # fused gate+up (2 groups of 130), int8
    (4, (384, 1003, 5, 4, 1, "from_quantized")),    # 4 ranks, ragged last shard
    (2, (256, 512, 1, 4, 2, "from_linear")),        # shard-then-quantize == quantize-then-shard
])
def test_sharded_matches_full_layer(world, case):
    res, codes = _run(world, case)
    assert len(res) == world, (res, codes)
    for rank, status, info in res:
        assert status == "ok", (rank, status, info)


@pytest.mark.parametrize("world,case", [
    (2, (256, 301, 6, 4, 1, "argmax")),             # uneven shards, int4
    (4, (128, 1003, 3, 8, 1, "argmax")),            # 4 ranks, int8
    (2, (256, 300, 4, 4, 1, "tie")),                # equal maxima in different shards -> smaller column
])
def test_sharded_argmax_matches_full_layer(world, case):
    """argmax through per-rank keys + all-gather of keys == argmax of the
    full layer's logits (ties to the smallest column, as torch.argmax)."""
    res, codes = _run(world, case)
    assert len(res) == world, (res, codes)
    for rank, status, info in res:
        assert status == "ok", (rank, status, info)


def test_dead_rank_raises_instead_of_hanging():
    res, codes = _run(2, (256, 128, 2, 4, 1, "die"), timeout=90)
    assert codes[1] == 3
    survivors = [r for r in res if r[0] == 0]
    assert survivors and survivors[0][1] == "error", res
