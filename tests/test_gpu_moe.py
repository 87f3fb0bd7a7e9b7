"""GPU parity of the sm_100a MoE layer against the CPU oracle and the
reference's golden outputs. Tolerances: expert ids and per-expert counts
bit-exact (near-ties within 4 ulps reported), bf16 output within
atol=rtol=1e-2 on >= 99.9% of elements."""
import numpy as np
import pytest
import torch

from conftest import cpu_weights, golden_activations, golden_cases, load_golden, oracle, pkg, workloads
from parity import check_output, check_routing, check_weights, run_gpu

pytestmark = pytest.mark.gpu

DEV = "cuda"
_W = {}


def gpu_weights(e_local=32, offset=0):
    key = (e_local, offset)
    if key not in _W:
        _W.clear()
        _W[key] = workloads().make_weights(e_local, offset, DEV, weight_seed=0)
    return _W[key]


def oracle_run(acts, w, scale=2.5, token_subset=None, offset=None):
    O = oracle()
    off = w.offset if offset is None else offset
    return O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden), acts.hidden_scale.numpy(),
                         lambda le: w.expert_cpu(le), off, scale, w.e_local, token_subset=token_subset)


@pytest.mark.parametrize("name", golden_cases())
def test_golden_reference_outputs(gpu_available, name):
    """Same inputs as the reference run that produced the fixture."""
    O = oracle()
    g = load_golden(name)
    acts = golden_activations(g)
    w = cpu_weights(int(g["offset"])).to(DEV)
    out, ids, wts, cnt = run_gpu(acts.to(DEV), w, float(g["scale"]))
    routing = O.route(acts.logits.numpy(), O.as_f32(acts.bias), float(g["scale"]))
    ties = check_routing(routing, ids, cnt, int(g["offset"]), 32)
    if not ties:
        np.testing.assert_array_equal(np.sort(ids.cpu().numpy(), axis=1), g["topk_idx_sorted"])
        np.testing.assert_array_equal(cnt.cpu().numpy(), g["counts"])
    check_output(out, O.bf16_bits_to_f32(g["out_bf16"]))


@pytest.mark.parametrize("T", [1, 2, 4, 8, 16, 32, 64, 256, 1024])
def test_parity_decode_and_mid(gpu_available, T):
    acts = workloads().config_activations(T)
    w = gpu_weights()
    out, ids, wts, cnt = run_gpu(acts.to(DEV), w)
    ref = oracle_run(acts, w)
    check_routing(ref["routing"], ids, cnt, 0, 32)
    check_weights(ref["routing"], ids, wts)
    check_output(out, ref["out_f32"])


def _rows_covering_every_mtile(T, e_local, counts, n_min, seed):
    """Tokens whose expert rows together touch every m-tile of every local
    expert (first, last and partial ones included), from the row placement of
    the call just made, topped up with random tokens to at least n_min."""
    rows_of = pkg().last_rows(T, e_local).cpu().numpy().astype(np.int64)
    ok = rows_of >= 0
    keys = (rows_of // 128)[ok]  # m-tile of each (token, local expert) row
    toks = np.broadcast_to(np.arange(T)[:, None], rows_of.shape)[ok]
    uniq, first = np.unique(keys, return_index=True)
    n_tiles = int(sum((int(c) + 127) // 128 for c in counts))
    assert len(uniq) == n_tiles, (len(uniq), n_tiles)
    rows = set(int(t) for t in toks[first])
    rng = np.random.default_rng(seed)
    for t in rng.permutation(T):
        if len(rows) >= n_min:
            break
        rows.add(int(t))
    return np.array(sorted(rows), dtype=np.int64)


@pytest.mark.parametrize("T", [4096, 8192, 16384])
def test_parity_skewed_prefill_every_mtile(gpu_available, T):
    """BASELINE configs[3] (4 hot local experts take every token). Routing and
    per-expert counts in full; the output on >= 512 tokens chosen so that
    every m-tile of every local expert (each expert's first and last, partial,
    tile included) contributes to some checked row. The oracle computes only
    those rows (each output row depends only on its own token)."""
    acts = workloads().config_activations(T)
    w = gpu_weights()
    out, ids, wts, cnt = run_gpu(acts.to(DEV), w)
    O = oracle()
    routing = O.route(acts.logits.numpy(), O.as_f32(acts.bias), 2.5)
    check_routing(routing, ids, cnt, 0, 32)
    counts = cnt.cpu().numpy()
    assert int(counts[:4].min()) > T // 2  # the 4 hot local experts take most tokens
    rows = _rows_covering_every_mtile(T, 32, counts, 512, T)
    assert len(rows) >= 512
    ref = oracle_run(acts, w, token_subset=rows)
    check_output(out, ref["out_f32"], rows=rows)


@pytest.mark.parametrize("T", [64, 100, 256])
def test_parity_one_local_expert_direct_combine(gpu_available, T):
    """Every token's only local expert is expert 3 (bias +16 on it, -8 on the
    other 31 local experts), so the call has one or two m-tiles: both GEMMs
    are split along K, and GEMM2 adds into per-token fp32 sums (the direct
    combine) with a full 64-row skinny tile (T=64, hi and lo in one MMA) and
    with 128-row tiles (T=100, 256). Routing, counts and every output row."""
    wl = workloads()
    a = wl.make_activations(T, seed=4242 + T)
    bias = a.bias.float()
    bias[:32] = -8.0
    bias[3] = 16.0
    acts = wl.Activations(a.logits, bias.to(torch.bfloat16), a.hidden, a.hidden_scale)
    w = gpu_weights()
    out, ids, wts, cnt = run_gpu(acts.to(DEV), w)
    counts = cnt.cpu().numpy()
    assert int(counts[3]) == T and int(counts.sum()) == T
    ref = oracle_run(acts, w)
    check_routing(ref["routing"], ids, cnt, 0, 32)
    check_weights(ref["routing"], ids, wts)
    check_output(out, ref["out_f32"])


def test_parity_beyond_benchmark_sizes_T65536(gpu_available):
    """Four times the largest benchmark call (near-uniform routing, ~16k
    local rows, a 13.5 GB workspace): 64-bit indexing of rows, scales and
    routing CTAs. Full routing/counts; output on a token subset. The
    workspace is released afterwards."""
    T = 65536
    acts = workloads().make_activations(T, seed=11)
    w = gpu_weights()
    out, ids, wts, cnt = run_gpu(acts.to(DEV), w)
    O = oracle()
    routing = O.route(acts.logits.numpy(), O.as_f32(acts.bias), 2.5)
    check_routing(routing, ids, cnt, 0, 32)
    rng = np.random.default_rng(T)
    rows = np.sort(np.concatenate([rng.choice(T, size=20, replace=False), [0, T - 1]]))
    ref = oracle_run(acts, w, token_subset=rows)
    check_output(out, ref["out_f32"], rows=rows)
    del out
    pkg().load().moe_fp8_ds_release_workspace()
    torch.cuda.empty_cache()


def test_cuda_graph_capture_and_replay(gpu_available):
    """The layer is graph-capturable once its workspace is sized: no host
    synchronisation or allocation inside the call. Replays on new input
    contents give the direct call's results."""
    m = pkg()
    w = gpu_weights()
    srcs = [workloads().config_activations(8).to(DEV), workloads().make_activations(8, seed=99).to(DEV)]
    refs = [run_gpu(x, w)[0] for x in srcs]
    st = workloads().make_activations(8, seed=1).to(DEV)   # static input buffers of the graph
    out = torch.empty((8, 7168), dtype=torch.bfloat16, device=DEV)

    def call():
        m.kernel(st.logits, st.bias, st.hidden, st.hidden_scale, w.w13, w.s13, w.w2, w.s2, 0, 2.5, out)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        call()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        call()
    for _ in range(2):
        for x, ref in zip(srcs, refs):
            for d, s_ in ((st.logits, x.logits), (st.bias, x.bias), (st.hidden, x.hidden),
                          (st.hidden_scale, x.hidden_scale)):
                d.copy_(s_)
            out.fill_(float("nan"))
            g.replay()
            torch.cuda.synchronize()
            diff = (out.float() - ref.float()).abs()
            assert torch.isfinite(out.float()).all()
            assert diff.max().item() <= 1e-2 * max(1.0, ref.float().abs().max().item())
    assert m.device_status() == 0
    del g


def test_no_local_tokens_gives_zero_output(gpu_available):
    acts = workloads().make_activations(16, seed=5)
    bias = acts.bias.float()
    bias[:32] -= 10.0  # no token can pick experts 0..31
    acts.bias = bias.to(torch.bfloat16)
    out, ids, wts, cnt = run_gpu(acts.to(DEV), gpu_weights())
    assert int(cnt.sum()) == 0
    assert torch.count_nonzero(out.float()).item() == 0


def test_offset_partial_range(gpu_available):
    """offset 240 with 32 local experts: only 240..255 exist (ref_moe.py:136)."""
    acts = workloads().make_activations(64, seed=11)
    w = gpu_weights()
    out, ids, wts, cnt = run_gpu(acts.to(DEV), w, offset=240)
    ref = oracle_run(acts, w, offset=240)
    check_routing(ref["routing"], ids, cnt, 240, 32)
    check_output(out, ref["out_f32"])


def test_zero_tokens_is_a_noop(gpu_available):
    m = pkg()
    w = gpu_weights()
    e = torch.empty
    m.kernel(e((0, 256), device=DEV), torch.zeros(256, dtype=torch.bfloat16, device=DEV),
             e((0, 7168), dtype=torch.float8_e4m3fn, device=DEV), e((56, 0), device=DEV),
             w.w13, w.s13, w.w2, w.s2, 0, 2.5, e((0, 7168), dtype=torch.bfloat16, device=DEV))
    torch.cuda.synchronize()


def test_repeated_and_resized_calls(gpu_available):
    """Workspace reuse: the self-resetting counters and accumulator give the
    same answer on repeated calls and after a larger call."""
    w = gpu_weights()
    a8 = workloads().config_activations(8).to(DEV)
    o1, i1, _, c1 = run_gpu(a8, w)
    run_gpu(workloads().config_activations(256).to(DEV), w)
    o2, i2, _, c2 = run_gpu(a8, w)
    assert torch.equal(i1, i2) and torch.equal(c1, c2)
    diff = (o1.float() - o2.float()).abs().max().item()
    assert diff <= 1e-2 * max(1.0, o1.float().abs().max().item())


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_devices_in_one_process(gpu_available):
    """One process drives the layer on two GPUs in turn: per-device workspace,
    launch attributes and tensor maps."""
    O = oracle()
    acts = workloads().config_activations(8)
    outs = []
    for d in (0, 1, 0):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            w = workloads().make_weights(32, 0, dev, weight_seed=0)
            out, ids, _, cnt = run_gpu(acts.to(dev), w)
        outs.append((out.cpu(), ids.cpu(), cnt.cpu()))
    ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden), acts.hidden_scale.numpy(),
                        lambda le: w.expert_cpu(le), 0, 2.5, 32)
    for out, ids, cnt in outs:
        check_output(out, ref["out_f32"])
        assert torch.equal(ids, outs[0][1]) and torch.equal(cnt, outs[0][2])


def test_route_entry(gpu_available):
    m = pkg()
    acts = workloads().make_activations(300, seed=3)
    ids, wts, cnt = m.route(acts.logits.to(DEV), acts.bias.to(DEV), 64, 32, 2.5)
    torch.cuda.synchronize()
    O = oracle()
    routing = O.route(acts.logits.numpy(), O.as_f32(acts.bias), 2.5)
    check_routing(routing, ids, cnt, 64, 32)
    check_weights(routing, ids, wts)


@pytest.mark.parametrize("e_local,offset", [(64, 64), (128, 0)])
def test_experts_entry_pre_routed(gpu_available, e_local, offset):
    """moe_fp8_ds_experts: rows arrive with their routing (expert-parallel owner side)."""
    m = pkg()
    O = oracle()
    acts = workloads().make_activations(96, seed=21)
    routing = O.route(acts.logits.numpy(), O.as_f32(acts.bias), 2.5)
    ids = torch.from_numpy(routing["topk_idx"].astype(np.int32))
    wts = torch.from_numpy(np.take_along_axis(routing["weights"], routing["topk_idx"], axis=1).astype(np.float32))
    w = gpu_weights(e_local, offset)
    out = torch.empty((96, 7168), dtype=torch.float32, device=DEV)
    m.experts(acts.hidden.to(DEV), acts.hidden_scale.to(DEV), ids.to(DEV), wts.to(DEV), w.w13, w.s13, w.w2, w.s2,
              offset, out)
    torch.cuda.synchronize()
    ref = O.moe_forward(acts.logits.numpy(), O.as_f32(acts.bias), O.as_u8(acts.hidden), acts.hidden_scale.numpy(),
                        lambda le: w.expert_cpu(le), offset, 2.5, e_local, routing=routing)
    got = out.cpu().numpy()
    frac = O.allclose_fraction(got, ref["out_f32"], 1e-2, 1e-2)
    assert frac >= 0.999, frac
