"""Host logic of the multi-GPU groups on CPU: shard arithmetic, expert ownership, operation tokens
and the exchange-region handshake over a real two-rank gloo process group (the CUDA calls are
replaced by a fake library)."""
from __future__ import annotations

import importlib
import os
import socket

import numpy as np
import pytest
import torch

Q4K, Q5K = 1, 4


@pytest.fixture(scope="module")
def gm(pkg):
    return importlib.import_module("minimax_rs_b200.group")


def test_tp_rows_split_whole_super_blocks(gm):
    assert gm.tp_rows(1536, 2, 0) == (0, 768) and gm.tp_rows(1536, 2, 1) == (768, 1536)
    with pytest.raises(ValueError):
        gm.tp_rows(1536, 4, 0)  # 384 is not a multiple of 256: the reason EP is used at W = 4 / 8


def test_tp_shards_recompose(gm, pkg):
    E, I, H = 3, 512, 512
    rng = np.random.default_rng(1)
    gate = torch.from_numpy(rng.integers(0, 256, E * I * pkg.row_bytes(Q4K, H), dtype=np.uint8))
    down = torch.from_numpy(rng.integers(0, 256, E * H * pkg.row_bytes(Q5K, I), dtype=np.uint8))
    g = [gm.tp_shard_gate_up(gate, E, I, H, Q4K, 2, r) for r in range(2)]
    d = [gm.tp_shard_down(down, E, H, I, Q5K, 2, r) for r in range(2)]
    assert g[0].shape == (E, I // 2, pkg.row_bytes(Q4K, H))
    assert torch.equal(torch.cat(g, dim=1).reshape(-1), gate)  # rows split along axis 1
    assert d[0].shape == (E, H, I // 2 // 256, 176)
    assert torch.equal(torch.cat(d, dim=2).reshape(-1), down)  # K split in whole super-blocks


def test_expert_ownership(gm):
    for w in (2, 4, 8):
        owned = [gm.ep_local_experts(256, w, r) for r in range(w)]
        assert sorted(sum(owned, [])) == list(range(256))
        assert all(len(o) == 256 // w for o in owned)
        assert all(gm.ep_owner(e, w) == r for r in range(w) for e in owned[r])


def test_token_counter_skips_zero(gm):
    t = gm.TokenCounter()
    assert [t.next() for _ in range(3)] == [1, 2, 3]
    t.value = 0xFFFFFFFF
    assert t.next() == 1  # 0 is reserved (flags start at zero)


def test_group_forward_draws_a_token_for_every_call(gm, monkeypatch):
    """Single-token calls take the group's next token like multi-token calls: the exchange flags
    and partial buffers are the group's, shared by every layer, so no two calls may share one."""
    seen = []

    class Lib:
        def mmrs_moe_block_forward_group(self, w, g, x, res, y, T, ids, wts, ws, nbytes, token, stream):
            seen.append((T, token))
            return 0

    class Layer:
        c = None

        def workspace(self, T):
            return torch.zeros(16, dtype=torch.uint8)

    class Stream:
        cuda_stream = 0

    monkeypatch.setattr(gm, "lib", lambda: Lib())
    monkeypatch.setattr(gm.C, "byref", lambda o: o)
    grp = gm.PeerGroup.__new__(gm.PeerGroup)
    grp.tokens, grp.c = gm.TokenCounter(), None
    layers = [Layer(), Layer(), Layer()]
    for t in range(6):
        T = 1 if t % 3 else 5
        grp.forward(layers[t % 3], torch.zeros(T, 8), y=torch.zeros(T, 8), stream=Stream())
    assert seen == [(5, 1), (1, 2), (1, 3), (5, 4), (1, 5), (1, 6)]


def test_numpy_kquant_expert_subset_matches_full_tensor(pkg):
    """The reference arm generates only the experts its tokens use; those windows must be the
    same bytes as in the whole synthetic tensor."""
    import importlib
    synth = importlib.import_module("minimax_rs_b200.synth")
    full = synth.kquant(Q5K, 7, 3, 6, 4, 512)
    sub = synth.kquant(Q5K, 7, 3, 6, 4, 512, expert_ids=[4, 1])
    assert np.array_equal(sub, full[[4, 1]])


class _FakeLib:
    """Stands in for the CUDA entry points PeerGroup uses."""

    def __init__(self, rank):
        self.rank = rank
        self.opened, self.closed, self.freed = [], [], []

    def mmrs_xch_bytes(self, cap):
        return 12288 + 8 * 8192 + 8 * cap

    def mmrs_peer_alloc(self, nbytes, out):
        out._obj.value = 0x100000 * (self.rank + 1)
        return 0

    def mmrs_ipc_handle(self, ptr, h):
        for i in range(64):
            h[i] = (self.rank * 7 + i) & 0xFF
        return 0

    def mmrs_ipc_open(self, h, out):
        owner = h[0] // 7
        out._obj.value = 0x7000000 + 0x1000 * owner
        self.opened.append(owner)
        return 0

    def mmrs_ipc_close(self, p):
        self.closed.append(p.value)
        return 0

    def mmrs_peer_free(self, p):
        self.freed.append(p.value)
        return 0


def _rank_main(rank, world, port, q):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import __graft_entry__ as ge
    import torch.distributed as dist
    ge.load_package()
    g = importlib.import_module("minimax_rs_b200.group")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fake = _FakeLib(rank)
    g.lib = lambda: fake

    def allgather(obj):
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    grp = g.PeerGroup(world, rank, ar_capacity=1024, expert_parallel=True, allgather=allgather)
    peers = [grp.c.peers[r] for r in range(world)]
    toks = [grp.tokens.next() for _ in range(3)]
    grp.close()
    q.put((rank, peers, fake.opened, toks, grp.c.world, grp.c.rank, grp.c.expert_parallel, fake.freed))
    dist.destroy_process_group()


def test_peer_group_handshake_gloo():
    import torch.multiprocessing as mp
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, peers, opened, toks, w, rk, ep, freed in results:
        assert (w, rk, ep) == (world, rank, 1)
        for r in range(world):
            expect = 0x100000 * (rank + 1) if r == rank else 0x7000000 + 0x1000 * r
            assert peers[r] == expect  # own region at its own index, peers' mappings in rank order
        assert opened == [r for r in range(world) if r != rank]
        assert toks == [1, 2, 3]
        assert freed == [0x100000 * (rank + 1)]


def test_group_forward_host_shares_the_token_sequence(gm, monkeypatch):
    """The host-buffer form of the group block draws from the same monotonic token counter as the
    device form, so the two may be mixed on one group without two calls sharing a token."""
    seen = []

    class Lib:
        def mmrs_moe_block_forward_group(self, w, g, x, res, y, T, ids, wts, ws, nbytes, token, stream):
            seen.append(("dev", T, token))
            return 0

        def mmrs_moe_block_forward_group_host(self, w, g, xh, res, yh, T, xd, yd, ids, wts, ws, nbytes, token,
                                              stream):
            seen.append(("host", T, token))
            return 0

    class Layer:
        c = None

        def workspace(self, T):
            return torch.zeros(16, dtype=torch.uint8)

    class Stream:
        cuda_stream = 0

    monkeypatch.setattr(gm, "lib", lambda: Lib())
    monkeypatch.setattr(gm.C, "byref", lambda o: o)
    grp = gm.PeerGroup.__new__(gm.PeerGroup)
    grp.tokens, grp.c = gm.TokenCounter(), None
    L = Layer()
    x, y = torch.zeros(1, 8), torch.zeros(1, 8)
    grp.forward(L, x, y=y, stream=Stream())
    grp.forward_host(L, x, y, x, y, stream=Stream())
    grp.forward_host(L, torch.zeros(3, 8), torch.zeros(3, 8), x, y, stream=Stream())
    grp.forward(L, x, y=y, stream=Stream())
    assert seen == [("dev", 1, 1), ("host", 1, 2), ("host", 3, 3), ("dev", 1, 4)]
