"""Host logic of the multi-GPU plans, on CPU with gloo ranks (world size 2).

The tensor-parallel test runs the exact step sequence of TensorParallelTransformer.forward with
fp32 torch ops in place of the kernels, on each rank's weight shards from tp_shard_state, with the
partial sums all-reduced over gloo, and checks the result against the full fp32 oracle.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from oracle import reference_fp32 as oracle
from tiktoktechjam2026track3_b200.cases import TransformerConfig
from tiktoktechjam2026track3_b200.sharding import batch_shard, cp_chunks, rs_rows, tp_check, tp_shard_state


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("batch,world", [(8, 1), (8, 2), (32, 8), (7, 3), (2, 4), (1, 8)])
def test_batch_shard_partitions_the_batch(batch, world):
    spans = [batch_shard(batch, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == batch
    for (a0, a1), (b0, _) in zip(spans, spans[1:]):
        assert a1 == b0
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1


def test_tp_check_rejects_uneven_splits():
    tp_check(TransformerConfig(1, 128, 2048, 16, 8192, 2, True), 8)
    with pytest.raises(ValueError):
        tp_check(TransformerConfig(1, 128, 768, 12, 3072, 2, True), 8)


def test_tp_shards_cover_the_weights():
    cfg = TransformerConfig(1, 16, 256, 4, 512, 1, True)
    state = oracle.build_reference_state(cfg, 0)
    shards = [tp_shard_state(state, cfg, 2, r)[0] for r in range(2)]
    q = state["layers.0.attention.q_proj.weight"]
    assert torch.equal(torch.cat([s["w_qkv"][:128] for s in shards], 0), q)
    assert torch.equal(torch.cat([s["w_o"] for s in shards], 1), state["layers.0.attention.out_proj.weight"])
    assert torch.equal(torch.cat([s["w_1"] for s in shards], 0), state["layers.0.ffn_in.weight"])
    assert torch.equal(torch.cat([s["w_2"] for s in shards], 1), state["layers.0.ffn_out.weight"])


def _tp_rank(rank, world, port, cfg, pad, result_queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        state = oracle.build_reference_state(cfg, 0)
        x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, 3, pad)
        shards = tp_shard_state(state, cfg, world, rank)
        h_loc, hd = cfg.num_heads // world, cfg.d_model // cfg.num_heads
        d_loc = h_loc * hd
        b, s, d = x.shape
        m = mask.reshape(-1, 1)

        def ln(t, w, bb):
            return F.layer_norm(t, (d,), w, bb, 1e-5)

        resid = x.reshape(-1, d).clone()
        y = ln(resid, shards[0]["ln1_w"], shards[0]["ln1_b"])
        for i, sh in enumerate(shards):
            qkv = y @ sh["w_qkv"].T + sh["b_qkv"]
            q, k, v = (qkv[:, j * d_loc:(j + 1) * d_loc].reshape(b, s, h_loc, hd).transpose(1, 2) for j in range(3))
            ctx = oracle.attention_core(q, k, v, mask, cfg.causal, hd**-0.5).transpose(1, 2).reshape(-1, d_loc)
            part = ctx @ sh["w_o"].T
            dist.all_reduce(part)
            resid = torch.where(m, resid + part + sh["b_o"], resid)
            y = ln(resid, sh["ln2_w"], sh["ln2_b"])
            part = F.gelu(y @ sh["w_1"].T + sh["b_1"]) @ sh["w_2"].T
            dist.all_reduce(part)
            resid = torch.where(m, resid + part + sh["b_2"], torch.zeros_like(resid))
            last = i == len(shards) - 1
            if last:
                y = torch.where(m, ln(resid, state["final_norm.weight"], state["final_norm.bias"]), 0.0)
            else:
                y = ln(resid, shards[i + 1]["ln1_w"], shards[i + 1]["ln1_b"])
        ref = oracle.forward(state, cfg, x, mask)
        result_queue.put((rank, float((y.reshape(b, s, d) - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pad", [0.0, 0.4])
def test_tensor_parallel_math_matches_full_model_over_gloo(pad):
    cfg = TransformerConfig(2, 40, 256, 4, 512, 2, True)
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_rank, args=(r, world, port, cfg, pad, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 1e-4, errs


@pytest.mark.parametrize("tokens,world", [(80, 2), (81, 2), (7, 3), (1, 4), (32768, 8)])
def test_rs_rows_partition_the_tokens(tokens, world):
    spans = [rs_rows(tokens, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == tokens
    for (a0, a1, per), (b0, _, _) in zip(spans, spans[1:]):
        assert a1 == b0 and a1 - a0 <= per
    per = spans[0][2]
    for row in range(tokens):  # the GEMM epilogue's owner rule agrees with the spans
        owner = min(row // per, world - 1)
        assert spans[owner][0] <= row < spans[owner][1]


@pytest.mark.parametrize("seq_len,world", [(32768, 2), (32768, 4), (32768, 8), (1024, 2)])
def test_cp_chunks_cover_the_sequence_with_equal_causal_work(seq_len, world):
    chunk, _ = cp_chunks(seq_len, world, 0)
    owned = sorted(c for r in range(world) for c in cp_chunks(seq_len, world, r)[1])
    assert owned == list(range(2 * world)) and chunk * 2 * world == seq_len
    # causal work of chunk c is proportional to (c + 1/2): every rank's pair sums to the same
    work = {sum(c + 0.5 for c in cp_chunks(seq_len, world, r)[1]) for r in range(world)}
    assert len(work) == 1
    with pytest.raises(ValueError):
        cp_chunks(1000, 2, 0)


def _rs_rank(rank, world, port, cfg, pad, result_queue):
    """The "rs" plan's step sequence (TensorParallelTransformer._forward_rs) with fp32 torch ops:
    partial rows reduced onto their owners (bias on rank 0), LayerNorm of the owned rows only,
    rows gathered to every rank."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        state = oracle.build_reference_state(cfg, 0)
        x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, 3, pad)
        shards = tp_shard_state(state, cfg, world, rank)
        h_loc, hd = cfg.num_heads // world, cfg.d_model // cfg.num_heads
        d_loc = h_loc * hd
        b, s, d = x.shape
        tokens = b * s
        spans = [rs_rows(tokens, world, r) for r in range(world)]
        r0, r1, _ = spans[rank]
        m = mask.reshape(-1, 1)
        lead = rank == 0

        def ln(t, w, bb):
            return F.layer_norm(t, (d,), w, bb, 1e-5)

        def reduce_to_owners(part):  # every rank's partial rows summed onto the row owner
            dist.all_reduce(part)  # (gloo has no reduce-scatter of uneven rows)
            return part[r0:r1]

        def gather_rows(rows_local):  # gloo gathers equal sizes: pad to rows_per_rank, then trim
            per = spans[0][2]
            padded = torch.zeros(per, d)
            padded[: rows_local.shape[0]] = rows_local
            out = [torch.zeros(per, d) for _ in range(world)]
            dist.all_gather(out, padded)
            return torch.cat([o[: spans[r][1] - spans[r][0]] for r, o in enumerate(out)], 0)

        resid = x.reshape(-1, d).clone()[r0:r1]  # this rank's rows of the residual
        y = ln(x.reshape(-1, d), shards[0]["ln1_w"], shards[0]["ln1_b"])  # first LayerNorm: all rows
        mine = m[r0:r1]
        for i, sh in enumerate(shards):
            qkv = y @ sh["w_qkv"].T + sh["b_qkv"]
            q, k, v = (qkv[:, j * d_loc:(j + 1) * d_loc].reshape(b, s, h_loc, hd).transpose(1, 2) for j in range(3))
            ctx = oracle.attention_core(q, k, v, mask, cfg.causal, hd**-0.5).transpose(1, 2).reshape(-1, d_loc)
            part = ctx @ sh["w_o"].T + (sh["b_o"] if lead else 0.0)
            resid = torch.where(mine, resid + reduce_to_owners(torch.where(m, part, 0.0)), resid)
            y = gather_rows(ln(resid, sh["ln2_w"], sh["ln2_b"]))
            part = F.gelu(y @ sh["w_1"].T + sh["b_1"]) @ sh["w_2"].T + (sh["b_2"] if lead else 0.0)
            resid = torch.where(mine, resid + reduce_to_owners(torch.where(m, part, 0.0)), torch.zeros_like(resid))
            last = i == len(shards) - 1
            if last:
                y = gather_rows(torch.where(mine, ln(resid, state["final_norm.weight"], state["final_norm.bias"]), 0.0))
            else:
                y = gather_rows(ln(resid, shards[i + 1]["ln1_w"], shards[i + 1]["ln1_b"]))
        ref = oracle.forward(state, cfg, x, mask)
        result_queue.put((rank, float((y.reshape(b, s, d) - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pad,world", [(0.0, 2), (0.4, 2), (0.4, 3)])
def test_reduce_scatter_plan_matches_full_model_over_gloo(pad, world):
    cfg = TransformerConfig(2, 41, 384, 6, 768, 2, True)  # 82 tokens: uneven row split
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rs_rank, args=(r, world, port, cfg, pad, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 1e-4, errs


def _cp_rank(rank, world, port, cfg, pad, result_queue):
    """The context-parallel plan's step sequence (ContextParallelTransformer.forward) with fp32
    torch ops: LayerNorms and GEMMs on this rank's zigzag chunks only, K/V rows all-gathered, the
    attention of this rank's query rows against every key (absolute causal positions)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        state = oracle.build_reference_state(cfg, 0)
        x, mask = oracle.generate_random_case(cfg, torch.device("cpu"), torch.float32, 3, pad)
        b, s, d = x.shape
        h, hd = cfg.num_heads, cfg.d_model // cfg.num_heads
        chunk, mine = cp_chunks(s, world, rank)
        idx = torch.cat([torch.arange(bb * s + c * chunk, bb * s + (c + 1) * chunk) for bb in range(b) for c in mine])

        def lin(t, name):
            return t @ state[f"{name}.weight"].T + state[f"{name}.bias"]

        def ln(t, name):
            return F.layer_norm(t, (d,), state[f"{name}.weight"], state[f"{name}.bias"], 1e-5)

        m_loc = mask.reshape(-1)[idx].reshape(-1, 1)
        resid = x.reshape(-1, d)[idx].clone()
        key_pos = torch.arange(s)
        for i in range(cfg.num_layers):
            p = f"layers.{i}"
            y = ln(resid, f"{p}.norm1")
            q_loc = lin(y, f"{p}.attention.q_proj")
            kv_loc = torch.cat([lin(y, f"{p}.attention.k_proj"), lin(y, f"{p}.attention.v_proj")], 1)
            gathered = [torch.zeros_like(kv_loc) for _ in range(world)]
            dist.all_gather(gathered, kv_loc)  # every rank's K/V rows
            kv = torch.zeros(b * s, 2 * d)
            for r in range(world):
                ch_r, mine_r = cp_chunks(s, world, r)
                idx_r = torch.cat([torch.arange(bb * s + c * ch_r, bb * s + (c + 1) * ch_r)
                                   for bb in range(b) for c in mine_r])
                kv[idx_r] = gathered[r]
            k = kv[:, :d].view(b, s, h, hd).transpose(1, 2)
            v = kv[:, d:].view(b, s, h, hd).transpose(1, 2)
            ctx = torch.zeros(b * s, d)
            qpos = idx % s
            qb = idx // s
            qh = q_loc.view(-1, h, hd)
            for n_row in range(idx.numel()):  # one query row at a time, absolute causal position
                bb, qq = int(qb[n_row]), int(qpos[n_row])
                sc = torch.einsum("hd,hkd->hk", qh[n_row], k[bb]) * hd**-0.5
                hidden = key_pos > qq if cfg.causal else torch.zeros(s, dtype=torch.bool)
                hidden = hidden | ~mask[bb]
                sc = sc.masked_fill(hidden[None], float("-inf"))
                ctx[n_row] = torch.einsum("hk,hkd->hd", torch.softmax(sc, -1), v[bb]).reshape(-1)
            a = lin(ctx[: idx.numel()], f"{p}.attention.out_proj")
            resid = torch.where(m_loc, resid + a, resid)
            f = lin(F.gelu(lin(ln(resid, f"{p}.norm2"), f"{p}.ffn_in")), f"{p}.ffn_out")
            resid = torch.where(m_loc, resid + f, torch.zeros_like(resid))
        out_loc = torch.where(m_loc, ln(resid, "final_norm"), 0.0)
        ref = oracle.forward(state, cfg, x, mask).reshape(-1, d)[idx]
        result_queue.put((rank, float((out_loc - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pad,world", [(0.0, 2), (0.3, 2)])
def test_context_parallel_plan_matches_full_model_over_gloo(pad, world):
    cfg = TransformerConfig(2, 1024, 128, 2, 256, 2, True)  # chunks of 256 tokens
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_cp_rank, args=(r, world, port, cfg, pad, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(world))
    assert max(errs.values()) < 1e-4, errs


def _failing_rank(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    if rank == 1:
        raise RuntimeError("rank 1 fails between steps")
    t = torch.ones(4)
    dist.all_reduce(t)  # rank 0 must not hang: the process-group timeout ends it with an error


def test_a_failing_rank_surfaces_as_errors_not_a_hang():
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_rank, args=(r, world, port)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes[1] not in (0, None)
    assert codes[0] not in (0, None)
