"""Tensor-parallel sharding, host side (CPU, no GPU): the shard helpers against
the dense oracle, a TP=2 decoder layer composed from per-rank oracles (partial
o_proj / down outputs summed) against the unsharded oracle layer, the merge of
per-rank greedy picks, and the same layer step with the partials summed by a
world-size-2 gloo all-reduce."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import oracle
from tests.gpu_util import oracle_layer, oracle_shape
from torch2iron_b200 import synth
from torch2iron_b200 import tp as TP
from torch2iron_b200.config import QuantizedQwenConfig

CFG = QuantizedQwenConfig(vocab_size=512, emb_dim=256, n_layers=1, n_heads=4, n_kv_groups=2, head_dim=128,
                          hidden_dim=1024, rms_norm_eps=1e-6, rope_base=1e6)


def _dense(lin):
    return oracle.autogptq_linear_to_dense(lin.qweight, lin.qzeros, lin.scales)


def test_shard_helpers_match_dense_slices():
    g = torch.Generator().manual_seed(11)
    lin = synth.random_linear(512, 1024, g)
    full = _dense(lin)
    assert torch.equal(_dense(TP.shard_out(lin, 128, 384)), full[128:384])
    assert torch.equal(_dense(TP.shard_in(lin, 256, 768)), full[:, 256:768])
    with pytest.raises(ValueError):
        TP.shard_in(lin, 64, 512)           # not on a 128-wide group
    with pytest.raises(ValueError):
        TP.shard_out(lin, 4, 64)            # not 8-aligned (qzeros packs 8 columns per word)


def test_check_tp_rejects_uneven_splits():
    TP.check_tp(CFG, 2)
    with pytest.raises(ValueError):
        TP.check_tp(CFG, 4)                 # 4 q heads of 128 -> 128 q columns per rank (o_proj K < 256)
    with pytest.raises(ValueError):
        TP.check_tp(CFG, 3)


def _local_decoder(model, tp, rank, batch, ctx):
    lcfg = TP.local_config(CFG, tp)
    layer = TP.shard_layer(model["layers"][0], CFG, tp, rank)
    return oracle.OracleDecoder(oracle_shape(lcfg), [oracle_layer(layer, lcfg)], embed=model["embed"],
                                final_norm=model["final_norm"], lm_head=model["embed"], max_ctx=ctx, batch=batch)


def test_tp2_layer_matches_unsharded_oracle():
    model = synth.random_model(CFG, seed=5)
    B, ctx = 3, 64
    g = torch.Generator().manual_seed(6)
    x = torch.randn(B, CFG.emb_dim, generator=g)
    pos = torch.tensor([0, 17, 63])
    full = oracle.OracleDecoder(oracle_shape(CFG), [oracle_layer(model["layers"][0], CFG)], embed=model["embed"],
                                final_norm=model["final_norm"], lm_head=model["embed"], max_ctx=ctx, batch=B)
    # earlier positions in the caches: same random K/V on both sides
    for r in range(B):
        for p in range(int(pos[r])):
            k = torch.randn(CFG.n_kv_groups, CFG.head_dim, generator=g).to(torch.bfloat16)
            v = torch.randn(CFG.n_kv_groups, CFG.head_dim, generator=g).to(torch.bfloat16)
            full.k_cache[0][r, :, p], full.v_cache[0][r, :, p] = k, v
    ref = full.layer_step(0, x, pos)
    # TP=2: rank r owns kv head r -> its cache is the r-th kv slice of the full cache
    # (this step's K/V included: each rank's attention rewrites its own at pos)
    summer = lambda parts: parts[0] + parts[1]     # the all-reduce of 2 ranks
    decs = {r: _local_decoder(model, 2, r, B, ctx) for r in range(2)}
    for r in range(2):
        decs[r].k_cache[0][:] = full.k_cache[0][:, r:r + 1]
        decs[r].v_cache[0][:] = full.v_cache[0][:, r:r + 1]
    eps = CFG.rms_norm_eps
    lay0 = model["layers"][0]
    xn = oracle.rms_norm(x, lay0["input_layernorm"], eps)
    x1 = x + summer({r: decs[r].attention(0, decs[r].layers[0], xn, pos) for r in range(2)})
    h = oracle.rms_norm(x1, lay0["post_attention_layernorm"], eps)
    y = x1 + summer({r: decs[r].layers[0].down_proj(torch.nn.functional.silu(decs[r].layers[0].gate_proj(h))
                                                   * decs[r].layers[0].up_proj(h)) for r in range(2)})
    assert (y - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()
    # the sharded K/V written this step are the full oracle's, per kv head
    for r in range(2):
        for b in range(B):
            p = int(pos[b])
            assert torch.equal(decs[r].k_cache[0][b, 0, p], full.k_cache[0][b, r, p])


def test_merge_argmax_across_vocab_shards():
    g = torch.Generator().manual_seed(3)
    tp, B, v = 4, 5, 37
    logits = torch.randn(B, tp * v, generator=g)
    logits[0, 3] = logits[0, 2 * v + 1] = 9.0           # tie across shards: lowest global index wins
    logits[1, tp * v - 1] = 9.5                          # maximum in the last shard
    vals, idx = [], []
    for r in range(tp):
        sl = logits[:, r * v:(r + 1) * v]
        i = sl.argmax(dim=1)
        vals.append(sl.gather(1, i[:, None])[:, 0])
        idx.append(i.to(torch.int32))
    got = TP.merge_argmax(torch.stack(vals), torch.stack(idx), v)
    assert torch.equal(got.long(), logits.argmax(dim=1))


# ---- world-size-2 gloo: the row-parallel partials summed by all_reduce ----
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, out_q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = synth.random_model(CFG, seed=5)
        g = torch.Generator().manual_seed(9)
        x = torch.randn(2, CFG.emb_dim, generator=g)
        pos = torch.tensor([0, 0])
        dec = _local_decoder(model, world, rank, 2, 64)
        lay0 = model["layers"][0]
        xn = oracle.rms_norm(x, lay0["input_layernorm"], CFG.rms_norm_eps)
        part = dec.attention(0, dec.layers[0], xn, pos).contiguous()
        dist.all_reduce(part)
        out_q.put((rank, (x + part).numpy()))
    finally:
        dist.destroy_process_group()


def test_tp2_attention_partials_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    model = synth.random_model(CFG, seed=5)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, CFG.emb_dim, generator=g)
    full = oracle.OracleDecoder(oracle_shape(CFG), [oracle_layer(model["layers"][0], CFG)], embed=model["embed"],
                                final_norm=model["final_norm"], lm_head=model["embed"], max_ctx=64, batch=2)
    lay0 = model["layers"][0]
    ref = x + full.attention(0, full.layers[0], oracle.rms_norm(x, lay0["input_layernorm"], CFG.rms_norm_eps),
                             torch.tensor([0, 0]))
    for r in range(2):
        got = torch.from_numpy(res[r])
        assert (got - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()


def test_push_slots_pair_every_writer_with_its_reader():
    """Push collective addressing: what rank r writes into rank q's buffer is
    exactly the slot rank q reads as rank r's partial, for every pair."""
    world, slot = 8, 64 * 4096 * 2
    bases = [0x7F0000000000 + (q << 32) for q in range(world)]
    table = [TP.push_slots(bases, r, slot) for r in range(world)]
    for r in range(world):
        reads, pushes = table[r]
        assert len(reads) == world and len(pushes) == world - 1
        assert reads[r] == bases[r] + r * slot                 # its own slot, written locally
        peers = [q for q in range(world) if q != r]
        for q, addr in zip(peers, pushes):
            assert addr == table[q][0][r]                     # rank q reads it as rank r's partial
    assert TP.push_slots(bases[:1], 0, slot) == ([bases[0]], [])
    with pytest.raises(ValueError):
        TP.push_slots(bases, world, slot)
