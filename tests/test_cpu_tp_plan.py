"""The tensor-parallel shard plan (qwc_tp_shard_of) on CPU, with world_size-2 gloo ranks:
the ranks' shards partition the GDN heads, attention q heads and FFN rows, every rank's kv
heads are the ones its q heads read, and a head-separable layer sliced by the plan
(column-parallel input projection, per-head mixing, row-parallel output projection)
summed by an all-reduce equals the unsliced layer — the decomposition the GPU prefill
uses, with its all-reduce after out_proj / o_proj / down_proj."""
import json
import os
import tempfile

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden", "config_budget.json")


def _cfg(abi, name):
    with open(GOLDEN) as f:
        case = json.load(f)[name]
    path = os.path.join(tempfile.gettempdir(), f"qwc_tpplan_{name}_{os.getpid()}.json")
    with open(path, "w") as f:
        json.dump(case["config"], f)
    return abi.load_config(path)


def _rank_main(rank, world, port, name, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    import __graft_entry__
    abi = __graft_entry__.load_package().abi
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg(abi, name)
        sh = abi.tp_shard(cfg, rank, world)
        shards = [None] * world
        dist.all_gather_object(shards, sh)
        # head-separable layer: y = Wo . mix(Wi x), mixing within each v head only
        g = torch.Generator().manual_seed(0)
        H, VH, D = 64, cfg.gdn_v_heads, 8
        Wi = torch.randn(VH * D, H, generator=g, dtype=torch.float64)
        Wo = torch.randn(H, VH * D, generator=g, dtype=torch.float64)
        mixm = torch.randn(VH, D, D, generator=g, dtype=torch.float64)
        x = torch.randn(5, H, generator=g, dtype=torch.float64)
        full = (torch.einsum("hij,thj->thi", mixm, (x @ Wi.T).view(5, VH, D)).reshape(5, -1)) @ Wo.T
        v0, nv = sh["vh0"], sh["n_vh"]
        rows = slice(v0 * D, (v0 + nv) * D)
        local = torch.einsum("hij,thj->thi", mixm[v0:v0 + nv], (x @ Wi[rows].T).view(5, nv, D)).reshape(5, -1)
        part = local @ Wo[:, rows].T
        dist.all_reduce(part)
        err = float((part - full).abs().max())
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump({"shards": shards, "err": err}, f)
    finally:
        dist.destroy_process_group()


def _free_port():
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("name", ["qwen3.5-0.8b-shaped", "qwen3.5-2b-shaped"])
def test_shard_plan_partitions_and_all_reduce_reproduces_the_layer(pkg, name):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank_main, args=(world, _free_port(), name, d), nprocs=world, start_method="spawn")
        res = [json.load(open(os.path.join(d, f"rank{r}.json"))) for r in range(world)]
    cfg = _cfg(pkg.abi, name)
    shards = res[0]["shards"]
    assert res[1]["shards"] == shards
    for key, n, total in (("kh0", "n_kh", cfg.gdn_k_heads), ("vh0", "n_vh", cfg.gdn_v_heads),
                          ("q0", "n_q", cfg.attn_q_heads), ("i0", "n_i", cfg.ffn_intermediate)):
        covered = sorted(x for s in shards for x in range(s[key], s[key] + s[n]))
        assert covered == list(range(total)), key
    grp = cfg.attn_q_heads // cfg.attn_kv_heads
    for s in shards:
        needed = {q // grp for q in range(s["q0"], s["q0"] + s["n_q"])}
        assert needed == set(range(s["kv0"], s["kv0"] + s["n_kv"]))
    for r in res:
        assert r["err"] < 1e-9


@pytest.mark.parametrize("world", [4, 8])
def test_shard_plan_wider_groups(pkg, world):
    cfg = _cfg(pkg.abi, "qwen3.5-2b-shaped")
    shards = [pkg.abi.tp_shard(cfg, r, world) for r in range(world)]
    assert sorted(q for s in shards for q in range(s["q0"], s["q0"] + s["n_q"])) == list(range(cfg.attn_q_heads))
    grp = cfg.attn_q_heads // cfg.attn_kv_heads
    for s in shards:
        assert s["n_kv"] == 1 and s["kv0"] == s["q0"] // grp  # replicated kv head
        assert s["n_i"] % 64 == 0


def test_shard_plan_rejects_uneven_splits(pkg):
    cfg = _cfg(pkg.abi, "qwen3.5-0.8b-shaped")
    with pytest.raises(pkg.abi.QwcError):
        pkg.abi.tp_shard(cfg, 0, 3)
