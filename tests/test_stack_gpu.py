"""The whole layer stack on the B200 through the C ABI, against the CPU
oracle (and, for the golden cases, against outputs of the reference itself).

Gate: the organiser's elementwise rule (abs <= 2e-3 OR abs <= 2e-2*|ref|,
all finite) on every output element compared; bit-exact: padded rows are
exactly 0. Every BASELINE config at full size: c1, c2 (seeds 0-2), c3a and c3b whole;
c4 every valid element of all 64 rows (oracle per row on its valid prefix,
rows are independent); c5 runs the full B=16 x S=65536 batch on the GPU and
compares its shortest sequence over the whole valid length, plus
whole-output properties (finite, padded rows exactly 0).
"""
from __future__ import annotations

import pytest
import torch

import oracle
from golden_cases import CASE_NAMES, load_case
from parity_log import record
from techjam2026_b200.configs import WORKLOADS, generate_case, make_state_dict
from techjam2026_b200.dispatch import Plan
from techjam2026_b200.fused import FusedTransformer
from techjam2026_b200.numerics import check, padded_rows_exactly_zero

pytestmark = pytest.mark.gpu


def _model(cfg, sd, plan=None):
    m = FusedTransformer(cfg, plan)
    m.load_state_dict(sd, strict=True)
    return m.eval()


def _oracle(cfg, sd, x, mask, query_chunk=None):
    torch.set_num_threads(max(1, torch.get_num_threads()))
    return oracle.forward(sd, cfg.num_layers, cfg.num_heads, x, mask, causal=cfg.causal,
                          query_chunk=query_chunk)


def _assert_gate(ref, out, what):
    res = check(ref, out.cpu())
    print(f"{what}: {res}")
    assert res.passed, f"{what}: {res}"
    return res


@pytest.mark.parametrize("name", CASE_NAMES)
@pytest.mark.parametrize("graph", [False, True])
def test_golden_cases_match_reference_output(name, graph):
    case = load_case(name)
    cfg = case["cfg"]
    m = _model(cfg, case["state_dict"], Plan(cuda_graph=graph))
    x, mask = case["x"].cuda(), case["mask"].cuda()
    out = m(x, mask)
    torch.cuda.synchronize()
    _assert_gate(case["out"], out, f"golden {name} graph={graph}")
    assert padded_rows_exactly_zero(out, mask)


@pytest.mark.parametrize("wname,seed", [("c1", 0), ("c2", 0), ("c2", 1), ("c2", 2),
                                        ("c3a", 0), ("c3b", 0)])
def test_baseline_configs_full_size(wname, seed):
    w = WORKLOADS[wname]
    cfg = w.cfg
    sd = make_state_dict(cfg, seed)
    x, mask = generate_case(cfg, seed, w.padding_ratio, w.input_scale)
    m = _model(cfg, sd)
    out = m(x.cuda(), mask.cuda())
    torch.cuda.synchronize()
    ref = _oracle(cfg, sd, x, mask, query_chunk=256)
    res = _assert_gate(ref, out, f"{wname} seed {seed}")
    record(f"{wname} seed {seed} full batch", res)
    assert padded_rows_exactly_zero(out, mask)


def _prefix_length(mask_row: torch.Tensor) -> int:
    """Valid length of a prefix mask row (the generator's masks are prefixes)."""
    n = int(mask_row.sum())
    assert bool(mask_row[:n].all()) and not bool(mask_row[n:].any()), "mask is not a prefix"
    return n


def _oracle_rows(cfg, sd, x, mask, rows, query_chunk=None):
    """Oracle outputs of the listed batch rows, each run on its valid prefix.

    Exact for prefix masks: a valid row attends only to keys before its
    sequence end, and every other op is per row, so the padding tail changes
    no valid output (and the reference zeroes padded output rows, which the
    tests check on the GPU output itself)."""
    outs = []
    for b in rows:
        n = _prefix_length(mask[b])
        outs.append(_oracle(cfg, sd, x[b:b + 1, :n], mask[b:b + 1, :n], query_chunk)[0])
    return outs


def test_c4_heavy_padding_every_row():
    """c4 at full size (B=64, S=2048, lengths U[1, 2048], 4 layers) through the
    captured graph: every valid output element of all 64 rows against the
    oracle, compared in slices of 8 rows (rows are independent), and every
    padded row exactly zero."""
    w = WORKLOADS["c4"]
    cfg = w.cfg
    sd = make_state_dict(cfg, 0)
    x, mask = generate_case(cfg, 0, w.padding_ratio)
    m = _model(cfg, sd)
    out = m(x.cuda(), mask.cuda()).cpu()
    torch.cuda.synchronize()
    assert padded_rows_exactly_zero(out, mask)
    assert bool(torch.isfinite(out).all())
    refs, gots = [], []
    for b0 in range(0, cfg.batch_size, 8):
        rows = list(range(b0, b0 + 8))
        for b, ref in zip(rows, _oracle_rows(cfg, sd, x, mask, rows)):
            refs.append(ref)
            gots.append(out[b, :ref.shape[0]])
    ref, got = torch.cat(refs), torch.cat(gots)
    assert ref.shape[0] == int(mask.sum())
    res = _assert_gate(ref, got, f"c4 all 64 rows ({ref.shape[0]} valid tokens)")
    record(f"c4 full batch, {ref.shape[0]} valid tokens x {cfg.d_model}", res)
    m.release_buffers()


def test_c5_long_sequence_whole_shortest_row():
    """c5 at full size (B=16, S=65536, 2 layers) on the GPU; the shortest
    sequence of the batch compared with the oracle over its whole valid
    length (query-chunked exact attention on the CPU), every other row
    checked for finiteness and exactly-zero padding."""
    w = WORKLOADS["c5"]
    cfg = w.cfg
    sd = make_state_dict(cfg, 0)
    x, mask = generate_case(cfg, 0, w.padding_ratio)
    m = _model(cfg, sd, Plan(cuda_graph=False))
    out = m.eager_forward(x.cuda(), mask.cuda())
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out).all())
    assert padded_rows_exactly_zero(out, mask.cuda())
    lens = mask.sum(1)
    b = int(lens.argmin())
    got = out[b, :int(lens[b])].cpu()
    m.release_buffers()
    del out
    torch.cuda.empty_cache()
    ref = _oracle_rows(cfg, sd, x, mask, [b], query_chunk=512)[0]
    res = _assert_gate(ref, got, f"c5 sequence {b}, all {ref.shape[0]} tokens")
    record(f"c5 sequence {b} whole ({ref.shape[0]} tokens x {cfg.d_model})", res)


def test_batch_slicing_is_bit_exact():
    """No op mixes batch elements, and every kernel's arithmetic for a row is
    independent of which tile the row lands in: a sub-batch reproduces the
    full batch's rows bit for bit (the property the reference's batch
    slicing relies on, kernelforge/optimized.py:343-348)."""
    w = WORKLOADS["c2"]
    cfg = w.cfg
    sd = make_state_dict(cfg, 0)
    x, mask = generate_case(cfg, 0, w.padding_ratio)
    m = _model(cfg, sd, Plan(cuda_graph=False))
    full = m.eager_forward(x.cuda(), mask.cuda())
    part = m.eager_forward(x[3:6].cuda().contiguous(), mask[3:6].cuda().contiguous())
    torch.cuda.synchronize()
    assert torch.equal(full[3:6], part)


def test_graph_equals_eager_and_held_output_survives():
    case = load_case("mini_s333")
    cfg = case["cfg"]
    m = _model(cfg, case["state_dict"])
    x, mask = case["x"].cuda(), case["mask"].cuda()
    eager = m.eager_forward(x, mask)
    g1 = m(x, mask)
    x2 = x.flip(0).contiguous()
    mask2 = mask.flip(0).contiguous()
    g2 = m(x2, mask2)
    torch.cuda.synchronize()
    assert torch.equal(eager, g1)
    assert torch.equal(g2, m.eager_forward(x2, mask2))
    assert torch.equal(g1, eager), "a held output must not change after another replay"


def test_no_mask_and_unpadded_inputs():
    case = load_case("mini_nopad")
    cfg = case["cfg"]
    m = _model(cfg, case["state_dict"])
    out_none = m(case["x"].cuda(), None)
    out_mask = m(case["x"].cuda(), case["mask"].cuda())
    torch.cuda.synchronize()
    _assert_gate(case["out"], out_none, "no mask")
    assert torch.equal(out_none, out_mask)


def test_submission_entry_passes_the_gate():
    import submission
    case = load_case("c1")
    cfg = case["cfg"]
    ours = submission.UserOptimizedTransformer(cfg)
    ours.load_state_dict(case["state_dict"], strict=True)
    ours = ours.cuda().eval()
    with torch.inference_mode():
        out = ours(case["x"].cuda(), case["mask"].cuda())
    assert ours._impl is not None and not ours._failed, "fused path must be the one running"
    _assert_gate(case["out"], out, "submission c1")


def test_native_library_is_the_one_loaded():
    """The CUDA path ran through the in-tree libkf_sm100.so (no silent fallback)."""
    import os
    from techjam2026_b200 import _lib, build
    assert _lib._lib is not None
    maps = open(f"/proc/{os.getpid()}/maps", encoding="utf-8").read()
    assert build.LIB_PATH in maps
    assert _lib.lib().kf_device_status(0) == 0


def test_streamed_forward_packed_copies_handle_changing_lengths():
    """Valid-prefix copies: the serving loop moves only each row's valid
    prefix, yet every result equals the model's whole output bit for bit
    (padded rows exactly zero), also when the same host result buffers are
    reused while rows get longer and shorter, and for a mask that is not a
    prefix (which takes whole-tensor copies)."""
    from techjam2026_b200.serving import StreamedForward
    case = load_case("mini_s333")
    cfg = case["cfg"]
    m = _model(cfg, case["state_dict"])
    B, S = cfg.batch_size, cfg.seq_len
    g = torch.Generator().manual_seed(5)
    xs, masks = [], []
    for k in range(6):
        lens = torch.randint(0, S + 1, (B,), generator=g)
        if k == 3:
            lens[:] = S                                 # every row full length
        mask = torch.arange(S)[None, :] < lens[:, None]
        x = torch.randn(B, S, cfg.d_model, generator=g).masked_fill(~mask[..., None], 0)
        if k == 4:
            mask = mask.clone()
            mask[0, 0] = False                          # not a prefix: whole copies
        xs.append(x.pin_memory())
        masks.append(mask.pin_memory())
    pipe = StreamedForward(m, xs[0].cuda(), masks[0].cuda())
    assert pipe.packed
    assert StreamedForward.prefix_lengths(masks[4]) is None
    outs = [torch.full_like(xs[0], 9.0).pin_memory() for _ in range(2)]
    for rnd in range(2):
        sched = list(range(6)) if rnd == 0 else list(range(5, -1, -1))
        res = [outs[i % 2] for i in range(6)]
        for i, k in enumerate(sched):
            pipe.run([xs[k]], [masks[k]], [res[i]])
            torch.cuda.current_stream().synchronize()
            want = m(xs[k].cuda(), masks[k].cuda()).cpu()
            assert torch.equal(res[i], want), f"round {rnd} batch {k}"
    assert pipe.last_h2d_bytes > 0


@pytest.mark.parametrize("mask_dtype", [torch.bool, torch.float32])
def test_streamed_forward_matches_per_batch_calls(mask_dtype):
    """The serving loop (uploads and downloads on their own streams, double
    buffers) returns, batch for batch, exactly what calling the model on each
    batch returns, including when consecutive batches differ. A bool mask
    runs one graph per buffer slot bound to the upload and download buffers;
    a float mask takes the copying path."""
    from techjam2026_b200.serving import StreamedForward
    case = load_case("mini_s333")
    cfg = case["cfg"]
    m = _model(cfg, case["state_dict"])
    xs, masks = [], []
    for seed in range(5):
        x, mask = generate_case(cfg, 100 + seed, 0.5)
        xs.append(x.pin_memory())
        masks.append(mask.to(mask_dtype).pin_memory())
    pipe = StreamedForward(m, xs[0].cuda(), masks[0].cuda())
    assert (pipe.bound is not None) == (mask_dtype == torch.bool)
    outs = pipe(xs, masks)
    again = pipe(xs[::-1], masks[::-1])
    for k in range(5):
        ref = m(xs[k].cuda(), masks[k].cuda()).cpu()
        assert torch.equal(outs[k], ref), f"batch {k}"
        assert torch.equal(again[4 - k], ref), f"reversed batch {k}"


def test_batch_streaming_under_a_memory_budget_is_exact():
    """With a budget of three sequences the c2 batch runs in slices of 3, 3
    and 2 sequences (two captured graphs) and reproduces the whole-batch
    forward bit for bit (no op mixes batch elements)."""
    w = WORKLOADS["c2"]
    cfg = w.cfg
    sd = make_state_dict(cfg, 0)
    x, mask = generate_case(cfg, 0, w.padding_ratio)
    x, mask = x.cuda(), mask.cuda()
    whole = _model(cfg, sd)(x, mask)
    m = FusedTransformer(cfg, memory_budget_bytes=None)
    m.load_state_dict(sd, strict=True)
    m = m.cuda().eval()
    m.memory_budget_bytes = 3 * m.bytes_per_sequence(cfg.seq_len) + 1
    sliced = m(x, mask)
    torch.cuda.synchronize()
    assert m.slice_rows(cfg.batch_size, cfg.seq_len, x.device) == 3
    assert len(m._graphs) == 2
    assert torch.equal(sliced, whole)


def test_organiser_accuracy_trials():
    """The organiser harness's accuracy gate on c2: five trials with seeds
    1234..1238 (its default seed), each drawn by generate_random_case and
    compared elementwise with the fp32 reference layer, through the public
    drop-in module."""
    import submission
    w = WORKLOADS["c2"]
    cfg = w.cfg
    sd = make_state_dict(cfg, 0)
    ours = submission.UserOptimizedTransformer(cfg)
    ours.load_state_dict(sd, strict=True)
    ours = ours.cuda().eval()
    for trial in range(5):
        x, mask = generate_case(cfg, 1234 + trial, w.padding_ratio, w.input_scale)
        with torch.inference_mode():
            out = ours(x.cuda(), mask.cuda())
        assert ours._impl is not None and not ours._failed
        ref = _oracle(cfg, sd, x, mask, query_chunk=256)
        _assert_gate(ref, out, f"organiser trial {trial + 1}/5 (seed {1234 + trial})")


def test_stream_k_gemms_share_one_workspace_and_pass_the_gate():
    """Every GEMM on stream-K scheduling (four shapes sharing one workspace:
    partials at its start, counters at its end) through several forwards:
    the gate holds, results repeat bit for bit, padded rows stay zero."""
    import dataclasses
    from techjam2026_b200.dispatch import DEFAULT_PLAN
    w = WORKLOADS["c2"]
    cfg = dataclasses.replace(w.cfg, batch_size=4, num_layers=2)
    sd = make_state_dict(cfg, 3)
    x, mask = generate_case(cfg, 3, w.padding_ratio, w.input_scale)
    plan = dataclasses.replace(DEFAULT_PLAN, bn_qkv=128, bn_out=128, bn_ffn1=128, bn_ffn2=64,
                               sk_qkv=True, sk_out=True, sk_ffn1=True, sk_ffn2=True)
    m = _model(cfg, sd, plan)
    xd, md = x.cuda(), mask.cuda()
    first = m(xd, md)
    again = [m(xd, md) for _ in range(3)]
    torch.cuda.synchronize()
    assert _lib_status() == 0
    for o in again:
        assert torch.equal(o, first)
    ref = _oracle(cfg, sd, x, mask)
    _assert_gate(ref, first, "stream-K c2 (B=4, L=2)")
    assert padded_rows_exactly_zero(first, mask)


def _lib_status():
    from techjam2026_b200 import _lib
    return _lib.lib().kf_device_status(0)


@pytest.mark.parametrize("wname", ["c4", "c3b"])
def test_rows_longest_first_is_bit_identical(wname):
    """plan.order_rows (kf_batch_order + kf_flash_fwd_tf32_ordered) changes
    only the attention schedule: the forward is bit-identical with and
    without it, eager and graph, on ragged batches."""
    import dataclasses
    w = WORKLOADS[wname]
    cfg = dataclasses.replace(w.cfg, batch_size=6, num_layers=1)
    sd = make_state_dict(cfg, 5)
    x, mask = generate_case(cfg, 5, w.padding_ratio, w.input_scale)
    xd, md = x.cuda(), mask.cuda()
    outs = []
    for order_rows in (False, True):
        from techjam2026_b200.dispatch import DispatchTable, probe
        spec = probe()
        plan, _ = DispatchTable.load_for(spec).lookup(spec.arch, torch.float32, cfg)
        m = _model(cfg, sd, dataclasses.replace(plan, order_rows=order_rows))
        outs.append((m(xd, md).clone(), m.eager_forward(xd, md).clone()))
        m.release_buffers()
    torch.cuda.synchronize()
    assert _lib_status() == 0
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    assert padded_rows_exactly_zero(outs[1][0], mask)


@pytest.mark.parametrize("with_mask", [False, True])
def test_single_token_sequences(with_mask):
    """S = 1 (the reference's single-token case: attention returns V of the
    one key exactly): the stack passes the gate against the oracle, graph
    and eager agree bit for bit."""
    import dataclasses
    cfg = dataclasses.replace(WORKLOADS["c1"].cfg, batch_size=5, seq_len=1, num_layers=2)
    sd = make_state_dict(cfg, 11)
    x, mask = generate_case(cfg, 11, 0.5)
    mask = mask if with_mask else None
    m = _model(cfg, sd)
    xd = x.cuda()
    md = mask.cuda() if mask is not None else None
    out = m(xd, md)
    eager = m.eager_forward(xd, md)
    torch.cuda.synchronize()
    assert _lib_status() == 0
    assert torch.equal(out, eager)
    _assert_gate(_oracle(cfg, sd, x, mask), out, f"S=1 mask={with_mask}")


@pytest.mark.parametrize("wname,masks", [("c4", "prefix"), ("c3b", "prefix"), ("c2", "prefix"),
                                         ("c3a", "prefix"), ("c1", "prefix"), ("c2", "random")])
def test_packed_ffn_forward_is_bit_identical(wname, masks):
    """plan.packed_ffn runs FFN1 and FFN2 over the valid tokens packed into
    consecutive rows (kf_pack_rows, kf_ln_add_mask_rows): every row's
    arithmetic is unchanged, so the forward is bit-identical to the padded
    one, through the captured graph and eagerly, on ragged batches and on
    masks that are not prefixes."""
    import dataclasses
    from techjam2026_b200.dispatch import DispatchTable, probe
    w = WORKLOADS[wname]
    cfg = dataclasses.replace(w.cfg, batch_size=min(6, w.cfg.batch_size), num_layers=2)
    sd = make_state_dict(cfg, 9)
    x, mask = generate_case(cfg, 9, w.padding_ratio, w.input_scale)
    if masks == "random":
        g = torch.Generator().manual_seed(9)
        mask = torch.rand(mask.shape, generator=g) > 0.35
        mask[:, 0] = True
    xd, md = x.cuda(), mask.cuda()
    spec = probe()
    plan, _ = DispatchTable.load_for(spec).lookup(spec.arch, torch.float32, cfg)
    outs = []
    for packed in (False, True):
        m = _model(cfg, sd, dataclasses.replace(plan, packed_ffn=packed))
        outs.append((m(xd, md).clone(), m.eager_forward(xd, md).clone(), m(xd, md).clone()))
        m.release_buffers()
    torch.cuda.synchronize()
    assert _lib_status() == 0
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
    assert padded_rows_exactly_zero(outs[1][0], mask)


@pytest.mark.parametrize("wname", ["c4", "c3b", "c2", "c3a"])
def test_persistent_attention_forward_is_bit_identical(wname):
    """plan.attn_persistent (kf_attn_schedule + kf_flash_fwd_tf32_sched)
    changes only how attention is scheduled and that query tiles without a
    valid query are left unwritten (their rows are padding, masked by every
    consumer): the forward is bit-identical to the one-CTA-per-tile kernel,
    through the captured graph and eagerly, on ragged batches."""
    import dataclasses
    from techjam2026_b200.dispatch import DispatchTable, probe
    w = WORKLOADS[wname]
    cfg = dataclasses.replace(w.cfg, batch_size=6, num_layers=2)
    sd = make_state_dict(cfg, 7)
    x, mask = generate_case(cfg, 7, w.padding_ratio, w.input_scale)
    xd, md = x.cuda(), mask.cuda()
    spec = probe()
    plan, _ = DispatchTable.load_for(spec).lookup(spec.arch, torch.float32, cfg)
    outs = []
    for persistent in (False, True):
        m = _model(cfg, sd, dataclasses.replace(plan, attn_persistent=persistent))
        outs.append((m(xd, md).clone(), m.eager_forward(xd, md).clone(), m(xd, md).clone()))
        m.release_buffers()
    torch.cuda.synchronize()
    assert _lib_status() == 0
    for a, b in zip(outs[0], outs[1]):
        assert torch.equal(a, b)
    assert padded_rows_exactly_zero(outs[1][0], mask)
