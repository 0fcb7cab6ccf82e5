"""Expert-parallel GPU tests (2+ GPUs): one child process per GPU; rank r owns experts
[r*E/N, (r+1)*E/N) and receives the rows routed to them.  Both transports run: peer memory
(rows written straight into the owners' matrices and results pushed back into the sources'
return matrices — from inside the GEMMs on the tensor-core path, by separate kernels on the
decode path, the two mixing freely between ranks) and the NCCL send/recv exchange
(HYMOE_EP_TRANSPORT=nccl).

Every output row's arithmetic is independent of how rows are tiled, so when both runs use
the tensor-core path the expert-parallel output must be bit-identical to the single-GPU
forward of the same tokens; it is also checked against the oracle within the parity
tolerance.  Skipped with fewer than 2 GPUs.
"""
import multiprocessing as mp
import os

import numpy as np
import pytest

import oracle as O
from moe_cases import REL_L2_TOL, host_layer, rel_l2

pytestmark = pytest.mark.gpu

H, I, E, K, SEED, WT = 512, 256, 64, 8, 41, O.Q4_0


def _gpu_count() -> int:
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def _layer(orc):
    return host_layer(orc, SEED, 0, H, I, E, WT)


def _placement(world):
    """Balanced placement for the Zipf bias of call 0 (expected load ~ exp(bias))."""
    import hymoe
    return hymoe.balance_placement(list(np.exp(O.zipf_bias(SEED, E))), world)


NORM_W = (1.0 + 0.05 * np.cos(np.arange(H))).astype(np.float32)


def _ep_worker(rank, world, nccl_id, tokens, max_tokens, q, transport="p2p", place=None, pre_norm=False,
               drop=None):
    import sys
    os.environ["HYMOE_EP_TRANSPORT"] = transport
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "hunyuan-image-3-80b.cpp_b200"),
                    os.path.dirname(os.path.abspath(__file__))]
    try:
        import oracle as O2
        import hymoe
        orc = O2.Oracle()
        lay = host_layer(orc, SEED, 0, H, I, E, WT)
        el = E // world
        slot_of = place if place is not None else list(range(E))
        mine = {e for e in range(E) if slot_of[e] // el == rank}
        egu = [lay["egu"][e] if e in mine else None for e in range(E)]
        edn = [lay["edn"][e] if e in mine else None for e in range(E)]
        m = hymoe.MoE(H, I, E, K, 1, max_tokens, device=rank, ep_rank=rank,
                      ep_size=world, nccl_id=nccl_id)
        if place is not None:
            m.set_placement(0, place)
        m.load_layer(0, lay["router"], lay["sgu"], lay["sdn"], egu, edn, WT)
        if pre_norm:
            m.set_norm(0, NORM_W, 1e-5)
        if drop is not None:
            m.set_routing(drop=drop, min_capacity=1)
        outs = []
        for call, t in enumerate(tokens):
            x = O2.synth_x(orc, SEED + 100 * call + rank, t, H)
            bias = O2.zipf_bias(SEED + call, E)
            outs.append(m.forward_host(0, x, bias=bias, debug=True, resid="x" if pre_norm else None,
                                       pre_norm=pre_norm))
        m.close()
        q.put((rank, "ok", outs))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, f"error: {e!r}", None))


def _run_ep(world, tokens_per_rank, transport="p2p", place=None, pre_norm=False, max_tokens=None, drop=None):
    import hymoe
    nccl_id = hymoe.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    if max_tokens is None:
        max_tokens = max(16, max(max(t) for t in tokens_per_rank))  # job-wide bound
    procs = [ctx.Process(target=_ep_worker,
                         args=(r, world, nccl_id, tokens_per_rank[r], max_tokens, q, transport, place,
                               pre_norm, drop))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, status, outs = q.get(timeout=600)
        assert status == "ok", f"rank {rank}: {status}"
        res[rank] = outs
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["p2p", "nccl"])
@pytest.mark.parametrize("tokens,placed", [([[200, 3], [150, 0]], False), ([[64], [5]], False),
                                           ([[300], [300]], False), ([[200, 3], [150, 0]], True),
                                           ([[300], [300]], True),
                                           # one rank on the tensor-core path, the other on the
                                           # decode path in the same call, three calls in a row
                                           ([[200, 40, 300], [5, 300, 70]], False)])
def test_expert_parallel_matches_single_gpu_and_oracle(orc, tokens, placed, transport):
    """placed: experts on ranks by hymoe_balance_placement (not the contiguous split)."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    world = 2
    place = _placement(world) if placed else None
    if placed:
        assert place != list(range(E))
    res = _run_ep(world, tokens, transport, place)
    import hymoe
    lay = _layer(orc)
    ncalls = len(tokens[0])
    single = hymoe.MoE(H, I, E, K, 1, max(max(t) for t in tokens) + 16, device=0)
    single.load_layer(0, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], WT)
    for call in range(ncalls):
        bias = O.zipf_bias(SEED + call, E)
        for rank in range(world):
            t = tokens[rank][call]
            x = O.synth_x(orc, SEED + 100 * call + rank, t, H)
            ep_out = res[rank][call]
            ref = single.forward_host(0, x, bias=bias, debug=True)
            assert np.array_equal(ep_out["idx"], ref["idx"])
            # Same GEMM path on both sides (every call above the 64-row decode regime):
            # identical bits.  Otherwise the decode kernel and the tensor-core path sum the
            # same fp16 products in a different order, within the parity tolerance.
            if all(tokens[r][call] > 64 for r in range(world)):
                assert np.array_equal(ep_out["out"], ref["out"]), f"rank {rank} call {call}"
            elif t:
                assert rel_l2(ep_out["out"], ref["out"]) <= REL_L2_TOL
            if t:
                o = orc.moe_forward(x, lay["router"], lay["sgu_f"], lay["sdn_f"], lay["egu_f"],
                                    lay["edn_f"], K, I, bias=bias)
                assert rel_l2(ep_out["out"], o["out"]) <= REL_L2_TOL
    single.close()


@pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_expert_parallel_pipelined_host_calls(orc, transport):
    """A context with max_tokens >= 4096 runs every host-pointer call as max_tokens / 2048 token
    chunks on every rank (copies overlapping the compute; a rank's chunk may be empty), debug
    outputs included: the same bits as the single-GPU call where every chunk is on the
    tensor-core path, the parity tolerance otherwise."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    tokens = [[300, 0, 4096], [2100, 5, 130]]
    res = _run_ep(2, tokens, transport, max_tokens=4096)
    import hymoe
    lay = _layer(orc)
    single = hymoe.MoE(H, I, E, K, 1, 4096, device=0)
    single.load_layer(0, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], WT)
    for call in range(3):
        bias = O.zipf_bias(SEED + call, E)
        for rank in range(2):
            t = tokens[rank][call]
            x = O.synth_x(orc, SEED + 100 * call + rank, t, H)
            ref = single.forward_host(0, x, bias=bias, debug=True)
            got = res[rank][call]
            for k in ("idx", "w", "logits", "probs"):
                assert np.array_equal(got[k], ref[k]), (rank, call, k)
            if all(tokens[r][call] // 2 > 64 for r in range(2)):
                assert np.array_equal(got["out"], ref["out"]), f"rank {rank} call {call}"
            elif t:
                assert rel_l2(got["out"], ref["out"]) <= REL_L2_TOL
    single.close()


@pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_expert_parallel_pre_norm_matches_single_gpu(orc, transport):
    """HYMOE_PRE_NORM on every rank: the dispatched rows are the normalised ones, the residual
    the raw ones; bit-identical to the single-GPU call (all calls on the tensor-core path)."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    tokens = [[200], [130]]
    res = _run_ep(2, tokens, transport, pre_norm=True)
    import hymoe
    lay = _layer(orc)
    single = hymoe.MoE(H, I, E, K, 1, 216, device=0)
    single.load_layer(0, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], WT)
    single.set_norm(0, NORM_W, 1e-5)
    bias = O.zipf_bias(SEED, E)
    for rank in range(2):
        x = O.synth_x(orc, SEED + rank, tokens[rank][0], H)
        ref = single.forward_host(0, x, bias=bias, debug=True, resid="x", pre_norm=True)
        assert np.array_equal(res[rank][0]["idx"], ref["idx"])
        assert np.array_equal(res[rank][0]["out"], ref["out"]), f"rank {rank}"
    single.close()


@pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["p2p", "nccl"])
def test_expert_parallel_capacity_drops_over_the_job(orc, transport):
    """Capacity-limited routing (topkgating_full with drop_tokens, src/hunyuan_moe_full.cpp:205-305)
    across ranks: the capacity comes from the job's token count and the k-major priority runs
    over the job's tokens in rank order, so every rank's output equals the one-GPU call over the
    concatenated tokens (rank 0's first) with the same routing: the same selections and dropped
    pairs (weight 0), the same output bits when every rank is on the tensor-core path.  The
    second call has a rank without tokens, which still takes part in the count exchange."""
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    tokens = [[300, 0], [200, 180]]
    cf = 0.5
    res = _run_ep(2, tokens, transport, drop=cf)
    import hymoe
    lay = _layer(orc)
    single = hymoe.MoE(H, I, E, K, 1, 520, device=0)
    single.load_layer(0, lay["router"], lay["sgu"], lay["sdn"], lay["egu"], lay["edn"], WT)
    single.set_routing(drop=cf, min_capacity=1)
    dropped = 0
    for call in range(2):
        bias = O.zipf_bias(SEED + call, E)
        xs = [O.synth_x(orc, SEED + 100 * call + r, tokens[r][call], H) for r in range(2)]
        ref = single.forward_host(0, np.concatenate(xs), bias=bias, debug=True)
        t0 = 0
        for rank in range(2):
            t = tokens[rank][call]
            got = res[rank][call]
            for k in ("idx", "w"):
                assert np.array_equal(got[k], ref[k][t0:t0 + t]), (rank, call, k)
            # Bits when every rank is on the tensor-core path; a rank without tokens computes
            # the rows it receives on the decode kernels (another summation order): tolerance.
            if all(tokens[r][call] > 64 for r in range(2)):
                assert np.array_equal(got["out"], ref["out"][t0:t0 + t]), (rank, call)
            elif t:
                assert rel_l2(got["out"], ref["out"][t0:t0 + t]) <= REL_L2_TOL, (rank, call)
            dropped += int((got["w"] == 0).sum())
            t0 += t
    assert dropped > 0  # the capacity did bite
    single.close()


def _timeout_worker(rank, world, nccl_id, q, go):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "oracle"), os.path.join(root, "hunyuan-image-3-80b.cpp_b200"),
                    os.path.dirname(os.path.abspath(__file__))]
    os.environ["HYMOE_EP_TRANSPORT"] = "p2p"
    os.environ["HYMOE_EP_TIMEOUT_S"] = "2"
    try:
        import oracle as O2
        import hymoe
        orc = O2.Oracle()
        lay = host_layer(orc, SEED, 0, H, I, E, WT)
        el = E // world
        mine = range(rank * el, (rank + 1) * el)
        egu = [lay["egu"][e] if e in mine else None for e in range(E)]
        edn = [lay["edn"][e] if e in mine else None for e in range(E)]
        m = hymoe.MoE(H, I, E, K, 1, 32, device=rank, ep_rank=rank, ep_size=world, nccl_id=nccl_id)
        m.load_layer(0, lay["router"], lay["sgu"], lay["sdn"], egu, edn, WT)
        x = O2.synth_x(orc, SEED + rank, 20, H)
        m.forward_host(0, x)  # every rank takes part
        status = "ok"
        if rank == 0:
            # Rank 1 skips this call (no kernels of its own in flight): rank 0's bounded
            # device-side waits for rank 1's flags must run out and report a timeout.
            try:
                m.forward_host(0, x)
                status = "no error"
            except hymoe.HymoeError as e:
                status = "timeout" if e.status == hymoe.STATUS_TIMEOUT else f"status {e.status}"
            try:  # the context refuses further expert-parallel calls
                m.forward_host(0, x)
                status += " / accepted"
            except hymoe.HymoeError:
                pass
            go.set()
        else:
            go.wait(120)  # stay mapped until rank 0's failed call has returned
        m.close()
        q.put((rank, status))
    except Exception as e:
        q.put((rank, f"error: {e!r}"))


@pytest.mark.skipif(_gpu_count() < 2, reason="needs 2 GPUs")
def test_peer_transport_bounded_wait_reports_timeout():
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import hymoe
    nccl_id = hymoe.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q, go = ctx.Queue(), ctx.Event()
    procs = [ctx.Process(target=_timeout_worker, args=(r, 2, nccl_id, q, go)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert res[0] == "timeout", res
    assert res[1] == "ok", res
