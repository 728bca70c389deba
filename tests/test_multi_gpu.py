"""Multi-GPU MoE block (TP = 2 and expert parallel) and the peer collectives, driven from one
process with one rank per device.  Needs at least two GPUs (skipped otherwise)."""
from __future__ import annotations

import ctypes as C
import importlib

import numpy as np
import pytest

from moe_cases import make_layer

pytestmark = pytest.mark.gpu
Q4K, Q5K = 1, 4


def _ngpu():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


needs2 = pytest.mark.skipif(_ngpu() < 2, reason="needs two GPUs")


def _group_mod(pkg):
    return importlib.import_module("minimax_rs_b200.group")


def _oracle_block(orc, L, x, residual):
    return orc.moe_block(L["router"].cpu().numpy(), L["bias"].cpu().numpy(), L["gate"].cpu().numpy(),
                         L["up"].cpu().numpy(), L["down"].cpu().numpy(), L["gu_type"], L["dn_type"], x, residual)


def _rank_layers(pkg, gm, L, world, ep):
    """Per-rank MoeLayer on device r: TP shards (ep False) or full copies (ep True)."""
    import torch
    E, H, I = L["E"], L["H"], L["I"]
    layers = []
    for r in range(world):
        dev = torch.device("cuda", r)
        if ep:
            gate, up, down = L["gate"].to(dev), L["up"].to(dev), L["down"].to(dev)
        else:
            gate = gm.tp_shard_gate_up(L["gate"], E, I, H, L["gu_type"], world, r).to(dev)
            up = gm.tp_shard_gate_up(L["up"], E, I, H, L["gu_type"], world, r).to(dev)
            down = gm.tp_shard_down(L["down"], E, H, I, L["dn_type"], world, r).to(dev)
        layers.append(pkg.MoeLayer(L["router"].to(dev), L["bias"].to(dev), gate, up, down, L["gu_type"],
                                   L["dn_type"]))
    return layers


def _run_group(pkg, groups, layers, x, residual, T):
    import torch
    ys, streams = [], []
    for r, (g, lay) in enumerate(zip(groups, layers)):
        dev = torch.device("cuda", r)
        with torch.cuda.device(dev):
            s = torch.cuda.Stream(device=dev)
            xs = x.to(dev)
            rs = None if residual is None else residual.to(dev)
            lay.workspace(T)
            torch.cuda.synchronize(dev)
            y = g.forward(lay, xs, residual=rs, stream=s)
            ys.append(y)
            streams.append(s)
    for r, s in enumerate(streams):
        s.synchronize()
    for g in groups:
        with torch.cuda.device(g._device):
            assert g.status() == 0
    return [y.cpu().numpy() for y in ys]


@needs2
@pytest.mark.parametrize("ep", [False, True], ids=["tp2", "ep2"])
@pytest.mark.parametrize("T", [1, 40, 5])
def test_group_block_matches_oracle(pkg, synth, orc, ep, T):
    import torch
    gm = _group_mod(pkg)
    E, H, I = 16, 512, 512
    L = make_layer(pkg, synth, torch.device("cuda", 0), E, H, I, Q4K, Q5K, seed=3100 + T, T=T, x_scale=0.05)
    groups = gm.PeerGroup.local([0, 1], ar_capacity=T * H, expert_parallel=ep)
    layers = _rank_layers(pkg, gm, L, 2, ep)
    ys = _run_group(pkg, groups, layers, L["x"], L["residual"], T)
    assert np.array_equal(ys[0].view(np.uint32), ys[1].view(np.uint32))  # identical on both ranks
    ry, _, _ = _oracle_block(orc, L, L["x"].cpu().numpy(), L["residual"].cpu().numpy())
    res = L["residual"].cpu().numpy()
    moe, rmoe = ys[0] - res, ry - res
    assert np.linalg.norm(moe - rmoe) / np.linalg.norm(rmoe) < 1e-4


@needs2
def test_group_decode_repeated_tokens(pkg, synth, orc):
    """Twenty decode steps in a row on TP = 2 (exchange buffers double-buffered by token)."""
    import torch
    gm = _group_mod(pkg)
    E, H, I = 16, 512, 512
    T = 20
    L = make_layer(pkg, synth, torch.device("cuda", 0), E, H, I, Q4K, Q5K, seed=3300, T=T)
    groups = gm.PeerGroup.local([0, 1], ar_capacity=H, expert_parallel=False)
    layers = _rank_layers(pkg, gm, L, 2, False)
    outs = [[], []]
    xs = [L["x"].to(torch.device("cuda", r)) for r in range(2)]
    for t in range(T):
        for r in range(2):
            with torch.cuda.device(r):
                layers[r].workspace(1)
                outs[r].append(groups[r].forward(layers[r], xs[r][t:t + 1]))
    for r in range(2):
        torch.cuda.synchronize(r)
    y0 = torch.cat([o.cpu() for o in outs[0]]).numpy()
    y1 = torch.cat([o.cpu() for o in outs[1]]).numpy()
    assert np.array_equal(y0, y1)
    for t in (0, T - 1):
        ry, _, _ = _oracle_block(orc, L, L["x"][t:t + 1].cpu().numpy(), None)
        assert np.linalg.norm(y0[t] - ry[0]) / np.linalg.norm(ry[0]) < 1e-4


@needs2
@pytest.mark.parametrize("ep", [False, True], ids=["tp2", "ep2"])
def test_group_decode_layers_round_robin(pkg, synth, orc, ep):
    """Three layers, each with its own workspace, share one group and take turns for twelve decode
    tokens (as a model's layers do).  The exchange flags and partial buffers belong to the group,
    so every call must wait for the peers' rows of *this* call: each step is checked against the
    oracle and the ranks must agree bit for bit."""
    import torch
    gm = _group_mod(pkg)
    E, H, I, NL, T = 16, 512, 512, 3, 12
    Ls = [make_layer(pkg, synth, torch.device("cuda", 0), E, H, I, Q4K, Q5K, seed=3400 + l, layer=l, T=T)
          for l in range(NL)]
    groups = gm.PeerGroup.local([0, 1], ar_capacity=H, expert_parallel=ep)
    layers = [_rank_layers(pkg, gm, L, 2, ep) for L in Ls]  # [layer][rank]
    xs = [[L["x"].to(torch.device("cuda", r)) for r in range(2)] for L in Ls]
    res = [[L["residual"].to(torch.device("cuda", r)) for r in range(2)] for L in Ls]
    outs = []
    for t in range(T):
        l = t % NL
        step = []
        for r in range(2):
            with torch.cuda.device(r):
                layers[l][r].workspace(1)
                step.append(groups[r].forward(layers[l][r], xs[l][r][t:t + 1], residual=res[l][r][t:t + 1]))
        outs.append((l, t, step))
    for r in range(2):
        torch.cuda.synchronize(r)
    for g in groups:
        with torch.cuda.device(g._device):
            assert g.status() == 0
    for l in range(NL):
        for r in range(2):
            with torch.cuda.device(r):
                assert layers[l][r].status() == 0
    for l, t, (y0, y1) in outs:
        a, b = y0.cpu().numpy(), y1.cpu().numpy()
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), (l, t)
        L = Ls[l]
        ry, _, _ = _oracle_block(orc, L, L["x"][t:t + 1].cpu().numpy(), L["residual"][t:t + 1].cpu().numpy())
        rr = L["residual"][t:t + 1].cpu().numpy()
        assert np.linalg.norm((a - rr) - (ry - rr)) / np.linalg.norm(ry - rr) < 1e-4, (l, t)


@needs2
@pytest.mark.parametrize("ep", [False, True], ids=["tp2", "ep2"])
@pytest.mark.parametrize("T", [1, 5])
def test_group_forward_host_matches_device_form(pkg, synth, ep, T):
    """mmrs_moe_block_forward_group_host (x and y in pinned host memory, one call) gives the device
    form's output bit for bit, on two calls in a row."""
    import torch
    gm = _group_mod(pkg)
    E, H, I = 16, 512, 512
    L = make_layer(pkg, synth, torch.device("cuda", 0), E, H, I, Q4K, Q5K, seed=3600 + T, T=T, x_scale=0.05)
    groups = gm.PeerGroup.local([0, 1], ar_capacity=T * H, expert_parallel=ep)
    layers = _rank_layers(pkg, gm, L, 2, ep)
    xs = [L["x"].to(f"cuda:{r}") for r in range(2)]
    rs = [L["residual"].to(f"cuda:{r}") for r in range(2)]
    x_host = [L["x"].cpu().pin_memory() for _ in range(2)]
    y_host = [torch.empty(T, H, dtype=torch.float32).pin_memory() for _ in range(2)]
    x_dev = [torch.empty(T, H, dtype=torch.float32, device=f"cuda:{r}") for r in range(2)]
    y_dev = [torch.empty(T, H, dtype=torch.float32, device=f"cuda:{r}") for r in range(2)]
    for r in range(2):
        with torch.cuda.device(r):
            layers[r].workspace(T)
        torch.cuda.synchronize(r)
    for call in range(2):
        ref = []
        for r in range(2):
            with torch.cuda.device(r):
                ref.append(groups[r].forward(layers[r], xs[r], residual=rs[r]))
        for r in range(2):
            with torch.cuda.device(r):
                groups[r].forward_host(layers[r], x_host[r], y_host[r], x_dev[r], y_dev[r], residual=rs[r])
        for r in range(2):
            torch.cuda.synchronize(r)
        for g in groups:
            with torch.cuda.device(g._device):
                assert g.status() == 0
        for r in range(2):
            assert torch.equal(y_host[r].view(torch.int32), ref[r].cpu().view(torch.int32)), (call, r)
    for g in groups:
        g.close()


def _owner_counts(ids, world):
    return [sum(1 for e in ids if e % world == r) for r in range(world)]


@pytest.mark.parametrize("world", [4, 8], ids=["ep4", "ep8"])
def test_group_decode_full_size_ep(pkg, synth, orc, world):
    """Expert parallel at full size (E = 256, H = 3072, I = 1536) on `world` GPUs, for tokens
    chosen so that at least one rank owns none of the token's eight experts (that rank computes
    nothing and only contributes zero rows to the exchange)."""
    if _ngpu() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch
    from moe_cases import oracle_decode
    gm = _group_mod(pkg)
    E, H, I = 256, 3072, 1536
    T = 24
    L = make_layer(pkg, synth, torch.device("cuda", 0), E, H, I, Q4K, Q5K, seed=3500 + world, T=T)
    router, bias = L["router"].cpu().numpy(), L["bias"].cpu().numpy()
    xh = L["x"].cpu().numpy()
    picked = []
    for t in range(T):
        ids, _ = orc.route_topk(orc.router_logits(xh[t:t + 1], router), bias)
        if min(_owner_counts(ids[0].tolist(), world)) == 0:
            picked.append(t)
    assert picked, "no token leaves a rank without experts"
    picked = picked[:3]
    groups = gm.PeerGroup.local(list(range(world)), ar_capacity=H, expert_parallel=True)
    layers = _rank_layers(pkg, gm, L, world, True)
    # Inputs and workspaces go to every device before the first group launch: a copy from cuda:0
    # issued after rank 0's kernel would wait behind it on cuda:0's stream, while that kernel
    # waits for the rows of the ranks whose launches the copy holds up.
    xs = [L["x"].to(f"cuda:{r}") for r in range(world)]
    rs = [L["residual"].to(f"cuda:{r}") for r in range(world)]
    for r in range(world):
        with torch.cuda.device(r):
            layers[r].workspace(1)
        torch.cuda.synchronize(r)
    outs = []
    for t in picked:
        step = []
        for r in range(world):
            with torch.cuda.device(r):
                step.append(groups[r].forward(layers[r], xs[r][t:t + 1], residual=rs[r][t:t + 1]))
        outs.append((t, step))
    for r in range(world):
        torch.cuda.synchronize(r)
    for g in groups:
        with torch.cuda.device(g._device):
            assert g.status() == 0
    for t, ys in outs:
        got = [y.cpu().numpy() for y in ys]
        for r in range(1, world):
            assert np.array_equal(got[0].view(np.uint32), got[r].view(np.uint32)), (t, r)
        ry, _, _, _ = oracle_decode(orc, pkg, L, xh[t], L["residual"][t].cpu().numpy())
        rr = L["residual"][t].cpu().numpy()
        assert np.linalg.norm((got[0][0] - rr) - (ry - rr)) / np.linalg.norm(ry - rr) < 1e-4, t
    for g in groups:
        g.close()


@needs2
@pytest.mark.parametrize("count", [3 * 4096 + 17, 512 * 3072 + 13], ids=["one_shot", "two_shot"])
def test_peer_all_reduce(pkg, synth, count):
    """Rank-ordered sum + residual, bit-identical on every rank.  Messages of 512K floats or more
    take the two-shot path (reduce-scatter + all-gather) on 4 or more ranks."""
    import torch
    gm = _group_mod(pkg)
    world = min(_ngpu(), 4)
    groups = gm.PeerGroup.local(list(range(world)), ar_capacity=(count + 3) // 4 * 4, expert_parallel=False)
    res = synth.normal_f32(count, 77, 9, 1.0)
    parts = [synth.normal_f32(count, 77, 10 + r, 1.0) for r in range(world)]
    expect = parts[0].copy()
    for r in range(1, world):
        expect = (expect + parts[r]).astype(np.float32)
    expect = (expect + res).astype(np.float32)
    ys = []
    for step in range(3):  # several tokens: both buffers of the double buffer
        ys = []
        for r, g in enumerate(groups):
            with torch.cuda.device(r):
                y = torch.empty(count, device=f"cuda:{r}")
                rt = torch.from_numpy(res).to(f"cuda:{r}")
                g.all_reduce(lambda ptr, r=r: pkg.lib().mmrs_synth_normal_f32(ptr, count, 77, 10 + r, 1.0, 0, None),
                             count, residual=rt, y=y)
                ys.append(y)
        for r in range(world):
            torch.cuda.synchronize(r)
        for y in ys:
            assert np.array_equal(y.cpu().numpy(), expect)


@needs2
@pytest.mark.parametrize("with_norm", [False, True])
def test_reference_tp2_peer_all_reduce(pkg, synth, with_norm):
    """launch_tp2_peer_all_reduce_f32 (ffi.rs:505-518) on two devices, epoch 0 (self counter)."""
    import torch
    L = pkg.lib()
    for d, o in ((0, 1), (1, 0)):
        with torch.cuda.device(d):
            assert L.mmrs_peer_enable(o) == 0
    count = 3072
    local = [torch.from_numpy(synth.normal_f32(count, 88, r, 1.0)).to(f"cuda:{r}") for r in range(2)]
    resid = torch.from_numpy(synth.normal_f32(count, 88, 5, 1.0))
    normw = torch.from_numpy(np.abs(synth.normal_f32(count, 88, 6, 1.0)))
    sig = [torch.zeros(32, dtype=torch.int32, device=f"cuda:{r}") for r in range(2)]
    outs, norms, streams = [], [], []
    for step in range(2):
        outs, norms, streams = [], [], []
        for r in range(2):
            with torch.cuda.device(r):
                s = torch.cuda.Stream()
                out = torch.empty(count, device=f"cuda:{r}")
                nrm = torch.empty(count, device=f"cuda:{r}") if with_norm else None
                rr = resid.to(f"cuda:{r}")
                nw = normw.to(f"cuda:{r}")
                L.launch_tp2_peer_all_reduce_f32(local[r].data_ptr(), local[1 - r].data_ptr(), rr.data_ptr(),
                                                 nw.data_ptr(), out.data_ptr(),
                                                 nrm.data_ptr() if nrm is not None else None, sig[r].data_ptr(),
                                                 sig[1 - r].data_ptr(), 0, count, 1e-6, C.c_void_p(s.cuda_stream))
                assert pkg.last_error() == 0
                outs.append(out)
                norms.append(nrm)
                streams.append((s, rr, nw))
        for s, _, _ in streams:
            s.synchronize()
    a = (local[0].cpu().numpy() + local[1].cpu().numpy()).astype(np.float32) + resid.numpy()
    for r in range(2):
        assert np.array_equal(outs[r].cpu().numpy(), a.astype(np.float32))
        assert sig[r][3].item() == 0  # no timeout recorded
    if with_norm:
        scale = 1.0 / np.sqrt(np.mean(a.astype(np.float64) ** 2) + 1e-6)
        ref = a * scale * normw.numpy()
        for r in range(2):
            got = norms[r].cpu().numpy()
            assert np.max(np.abs(got - ref) / (np.abs(ref) + 1e-6)) < 1e-5
        assert np.array_equal(norms[0].cpu().numpy(), norms[1].cpu().numpy())


@needs2
def test_reference_tp2_peer_broadcast(pkg, synth):
    import torch
    L = pkg.lib()
    for d, o in ((0, 1), (1, 0)):
        with torch.cuda.device(d):
            assert L.mmrs_peer_enable(o) == 0
    count = 1000
    src = torch.from_numpy(synth.normal_f32(count, 89, 1, 1.0)).to("cuda:1")
    out0 = torch.zeros(count, device="cuda:0")
    sig = [torch.zeros(32, dtype=torch.int32, device=f"cuda:{r}") for r in range(2)]
    streams = []
    for r in range(2):
        with torch.cuda.device(r):
            s = torch.cuda.Stream()
            # rank 1 copies its source into rank 0's output (a peer pointer), as the reference uses it
            L.launch_tp2_peer_broadcast_f32(src.data_ptr() if r == 1 else None, out0.data_ptr(), sig[r].data_ptr(),
                                            sig[1 - r].data_ptr(), 7, r, count, C.c_void_p(s.cuda_stream))
            assert pkg.last_error() == 0
            streams.append(s)
    for s in streams:
        s.synchronize()
    assert np.array_equal(out0.cpu().numpy(), src.cpu().numpy())
