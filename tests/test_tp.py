"""Tensor parallelism: shard geometry on CPU ranks, and TP=2 decode on two GPUs.

CPU part: two `gloo` ranks each ask the library (host-only entry point, no device) for their
shard of several BASELINE shapes and all-gather them; the shards must tile every split
dimension exactly once.  GPU part (skipped with fewer than two GPUs): two spawned processes
load their shards of the tiny config, join one NCCL group and must reproduce the single-GPU
greedy tokens and logits, once with NCCL's all-reduce for the residual sums and once with the
peer-memory all-reduce (CUDA IPC handles exchanged through files), whose results must also equal
the NCCL run's bit for bit (with two ranks both add the same two partials).
"""
import json
import os
import socket
import tempfile
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from dotllm_b200 import synth

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _shard_rank(rank, world, port, configs, q):
    import torch.distributed as dist

    from dotllm_b200.engine import tp_shard

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        mine = {name: tp_shard(cfg, world, rank) for name, cfg in configs.items()}
        everyone = [None] * world
        dist.all_gather_object(everyone, mine)
        if rank == 0:
            q.put(everyone)
    finally:
        dist.destroy_process_group()


def _config_dict(cfg):
    return {"template_id": 0, "hidden": cfg.hidden, "layers": cfg.layers, "context": cfg.context,
            "vocab": cfg.vocab, "ffn": cfg.ffn, "heads": cfg.heads, "heads_kv": cfg.heads_kv,
            "head_dim": cfg.head_dim}


def test_tp_shards_tile_gloo():
    configs = {n: _config_dict(synth.get(n)) for n in ("tiny", "llama1b", "llama8b")}
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_shard_rank, args=(r, world, port, configs, q)) for r in range(world)]
    for p in procs:
        p.start()
    everyone = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for name, cfg in configs.items():
        hd = cfg["head_dim"]
        for lo, n, total in (("q_lo", "q_n", cfg["heads"] * hd), ("kv_lo", "kv_n", cfg["heads_kv"] * hd),
                             ("ffn_lo", "ffn_n", cfg["ffn"]), ("vocab_lo", "vocab_n", cfg["vocab"])):
            spans = sorted((r[name][lo], r[name][n]) for r in everyone)
            pos = 0
            for a, b in spans:
                assert a == pos and b > 0, (name, lo, spans)
                pos = a + b
            assert pos == total, (name, lo, spans, total)
        # column shards of attn_output / ffn_down fall on whole 256-weight super-blocks
        for r in everyone:
            assert r[name]["q_n"] % 256 == 0 and r[name]["ffn_n"] % 256 == 0


def test_tp_shard_rejects_uneven():
    from dotllm_b200.engine import tp_shard
    from dotllm_b200.native import CudaBackendError

    cfg = _config_dict(synth.get("tiny"))
    with pytest.raises(CudaBackendError):
        tp_shard(cfg, 3, 0)  # 8 heads / 4 kv heads do not split in 3
    with pytest.raises(CudaBackendError):
        tp_shard(cfg, 4, 0)  # 128-column attn_output shards are not whole super-blocks


def _exchange_files(m, rank, world, xdir):
    """Every rank writes its peer all-reduce handle to a file and opens all ranks' handles."""
    h = m.tp_exchange_handle()
    tmp = os.path.join(xdir, f"h{rank}.tmp")
    with open(tmp, "wb") as f:
        f.write(h)
    os.replace(tmp, os.path.join(xdir, f"h{rank}"))
    handles = []
    for r in range(world):
        fn = os.path.join(xdir, f"h{r}")
        t0 = time.time()
        while not os.path.exists(fn):
            assert time.time() - t0 < 120, "peer handle never arrived"
            time.sleep(0.05)
        handles.append(open(fn, "rb").read())
    m.tp_exchange_open(handles)


class _FakeExchange:
    """Stands in for a model's exchange entry points on CPU; `fail` names the call that raises."""

    def __init__(self, rank, fail=None):
        self.rank, self.fail, self.calls = rank, fail, []

    def tp_exchange_handle(self):
        self.calls.append("handle")
        if self.fail == "handle":
            raise RuntimeError(f"rank {self.rank}: export refused")
        return bytes([self.rank]) * 128

    def tp_exchange_open(self, handles):
        self.calls.append(("open", tuple(h[0] for h in handles)))
        if self.fail == "open":
            raise RuntimeError(f"rank {self.rank}: open refused")

    def tp_exchange_use(self, on):
        self.calls.append(("use", on))


def _open_peer_rank(rank, world, port, fail_rank, fail_call, q):
    import torch.distributed as dist

    from dotllm_b200.engine import tp_open_peer

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        m = _FakeExchange(rank, fail_call if rank == fail_rank else None)

        def gather(obj):
            got = [None] * world
            dist.all_gather_object(got, obj)
            return got

        why = tp_open_peer(m, gather)
        q.put((rank, why, m.calls))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank,fail_call", [(-1, None), (1, "handle"), (0, "open"), (2, "open")])
def test_tp_open_peer_agreement_gloo(fail_rank, fail_call):
    """Every rank ends with the same answer: the peer all-reduce on everywhere, or off everywhere
    (ranks whose own open succeeded turn it off again when another rank failed)."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_open_peer_rank, args=(r, world, port, fail_rank, fail_call, q))
             for r in range(world)]
    for p in procs:
        p.start()
    got = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    whys = {why for _, why, _ in got}
    assert len(whys) == 1
    why = whys.pop()
    if fail_rank < 0:
        assert why is None
        for rank, _, calls in got:
            assert calls == ["handle", ("open", (0, 1, 2))]
        return
    assert f"rank {fail_rank}" in why or "could not export" in why
    for rank, _, calls in got:
        opened = any(c[0] == "open" for c in calls if isinstance(c, tuple))
        if fail_call == "handle":
            assert not opened  # nobody opens an incomplete set of handles
            assert ("use", False) not in calls
        elif rank == fail_rank:
            assert calls[-1] == ("open", (0, 1, 2))  # its open raised: nothing to turn off
        else:
            assert calls[-1] == ("use", False)


def _tp_rank(rank, world, path, prompt, steps, q_in, q_out, xdir=None):
    from dotllm_b200.engine import CudaModel, tp_unique_id

    m = CudaModel.load_tp(path, world, rank, device=rank)
    if rank == 0:
        uid = tp_unique_id()
        for _ in range(world - 1):
            q_in.put(uid)
    else:
        uid = q_in.get(timeout=120)
    m.tp_init(uid)
    if xdir is not None:
        _exchange_files(m, rank, world, xdir)
    s = m.session(kv="f32")
    _, lg = s.prefill(prompt, want_logits=True)
    toks = s.generate(prompt, steps)
    # five sessions decoded together take the batched matmul path
    ss = [m.session(kv="f32") for _ in range(5)]
    firsts = [x.prefill(prompt)[0] for x in ss]
    from dotllm_b200.engine import decode_batch
    nxt, blg = decode_batch(ss, firsts, want_logits=True)
    if rank == 0:
        q_out.put((list(map(int, toks)), lg, firsts, list(map(int, nxt)), blg))
    s.close()
    for x in ss:
        x.close()
    m.close()


_NCCL_RUN = {}


@pytest.mark.gpu
@pytest.mark.parametrize("allreduce", ["nccl", "peer"])
def test_tp2_matches_single_gpu(gpu, allreduce):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from dotllm_b200.engine import CudaModel, decode_batch

    name = "tiny"
    cfg = synth.get(name)
    path = synth.build_model(cfg)
    prompt = synth.prompt_tokens(cfg)
    steps = 24
    ref = CudaModel.load(path)
    rs = ref.session(kv="f32")
    _, ref_lg = rs.prefill(prompt, want_logits=True)
    ref_toks = list(map(int, rs.generate(prompt, steps)))
    rss = [ref.session(kv="f32") for _ in range(5)]
    rf = [x.prefill(prompt)[0] for x in rss]
    ref_nxt, ref_blg = decode_batch(rss, rf, want_logits=True)
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    xdir = tempfile.mkdtemp(prefix="tpx") if allreduce == "peer" else None
    procs = [ctx.Process(target=_tp_rank, args=(r, 2, path, prompt, steps, q_in, q_out, xdir)) for r in range(2)]
    for p in procs:
        p.start()
    toks, lg, firsts, nxt, blg = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.abs(lg - ref_lg).max() < 1e-3
    assert toks == ref_toks
    assert firsts == [ref_toks[0]] * 5
    assert np.abs(blg - ref_blg).max() < 1e-3
    assert nxt == list(map(int, ref_nxt))
    golden = json.load(open(os.path.join(HERE, "golden", "greedy_tokens.json")))["tiny"]["tokens"]
    assert toks == golden[:steps]
    _NCCL_RUN.setdefault(allreduce, (lg, blg))
    if allreduce == "peer" and "nccl" in _NCCL_RUN:
        assert np.array_equal(lg, _NCCL_RUN["nccl"][0])
        assert np.array_equal(blg, _NCCL_RUN["nccl"][1])
