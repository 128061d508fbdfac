"""Multi-GPU plans on B200s (needs 2+ GPUs; skipped otherwise): one process per GPU over NCCL.

* tensor parallel (heads/FFN columns) agrees with the single-GPU model within the parity gate
  (reduction order differs, so not bitwise), both with the reduce-scatter fused into the GEMM
  epilogues and the all-gather into the LayerNorm ("rs") and with the NCCL all-reduce;
* context parallel (zigzag token chunks, K/V rows all-gathered over NVLink) agrees likewise;
* a batch shard on rank r is bit-identical to the same sequences of the single-GPU run.
"""

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import reference_fp32 as oracle
from tiktoktechjam2026track3_b200 import UserOptimizedTransformer, baseline_gate
from tiktoktechjam2026track3_b200.cases import TransformerConfig
from tiktoktechjam2026track3_b200.sharding import ContextParallelTransformer, TensorParallelTransformer, batch_shard

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg, pad, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        state = oracle.build_reference_state(cfg, 0)
        x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, 1, pad)
        xb, mask = x.to(dev, torch.bfloat16), mask.to(dev)
        model = UserOptimizedTransformer(cfg)
        model.load_state_dict(state, strict=True)
        model = model.to(device=dev, dtype=torch.bfloat16).eval()
        collectives = ["nccl", "rs", "cp"]
        with torch.inference_mode():
            single = model(xb, mask)
            b0, b1 = batch_shard(cfg.batch_size, world, rank)
            shard = model(xb[b0:b1].contiguous(), mask[b0:b1].contiguous())
            outs = {}
            for coll in collectives:
                tp = (ContextParallelTransformer(cfg, state, dev) if coll == "cp" else
                      TensorParallelTransformer(cfg, state, dev, collective=coll))
                outs[coll] = tp(xb, mask)
                outs[coll + "_again"] = tp(xb * 0.5, mask)
                outs[coll + "_again_ref"] = model(xb * 0.5, mask)
                torch.cuda.synchronize()
                tp.close()
                dist.barrier()
        torch.cuda.synchronize()
        from tiktoktechjam2026track3_b200 import _capi

        status = _capi.device_status(clear=True)
        result = {"rank": rank, "status": status, "shard_equal": bool(torch.equal(shard, single[b0:b1])),
                  "collectives": collectives}
        for coll in collectives:
            g = baseline_gate(outs[coll], single.float())
            g2 = baseline_gate(outs[coll + "_again"], outs[coll + "_again_ref"].float())
            result[coll] = (g.passed and g2.passed, g.normwise_error, g2.normwise_error,
                            bool(torch.all(outs[coll][~mask] == 0)))
        q.put(result)
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("pad", [0.0, 0.3])
def test_tensor_parallel_and_batch_shards_on_two_gpus(cuda_device, pad):
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip("needs 2 GPUs")
    cfg = TransformerConfig(2, 1024, 2048, 16, 8192, 2, True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg, pad, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = [q.get(timeout=5) for _ in range(world)]
    for r in results:
        assert r["status"] == 0, r
        assert r["shard_equal"], r
        for coll in r["collectives"]:
            assert r[coll][0], (coll, r)
            assert r[coll][3], (coll, r)  # padding rows are zero
