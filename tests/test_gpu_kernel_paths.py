"""Each CUDA kernel family (forced through the C ABI path knob) against the reference golden outputs.

``path="tensor"`` runs the tcgen05/TMEM kernel and ``path="decode"`` the warp-level kernel on every
golden case, whatever the query length, so both kernels are held to the reference on every head
dimension, page size, causal mode, length pattern and NaN-poisoned pool the fixtures cover.
"""
import pytest
import torch

from fixtures import build_case, dtype_name, oracle_output
from golden_data import entry_params, expected_bits, output_index
from oracle import dtype_bits_to_f32
from test_gpu_parity import _check, _run

pytestmark = pytest.mark.gpu

ENTRIES = output_index()


def test_tensor_path_smallest_case_first():
    inputs = build_case(("tiny_tensor", 1, 130, 1, 128, 128, 2), 7, torch.bfloat16, False, "full")
    out = _run(inputs, path="tensor")
    _check(out, oracle_output(inputs), inputs)


@pytest.mark.parametrize("path", ["tensor", "decode"])
@pytest.mark.parametrize("entry", ENTRIES, ids=[e["key"] for e in ENTRIES])
def test_kernel_path_matches_reference_golden(entry, path):
    case, seed, dtype, causal, pattern = entry_params(entry)
    inputs = build_case(case, seed, dtype, causal, pattern)
    expected = dtype_bits_to_f32(expected_bits(entry), dtype_name(dtype))
    _check(_run(inputs, path=path), expected, inputs)


@pytest.mark.parametrize("kernel", ["halves", "single"])
@pytest.mark.parametrize("entry", ENTRIES, ids=[e["key"] for e in ENTRIES])
def test_other_tensor_kernels_match_reference_golden(entry, kernel):
    # The key-halves kernel (head dims up to 128) and the one-tile kernel (every head dim) on every golden case.
    case, seed, dtype, causal, pattern = entry_params(entry)
    if kernel == "halves" and case[4] > 128:
        pytest.skip("the key-halves kernel serves head dims up to 128")
    inputs = build_case(case, seed, dtype, causal, pattern)
    expected = dtype_bits_to_f32(expected_bits(entry), dtype_name(dtype))
    _check(_run(inputs, path="tensor", tensor_kernel=kernel), expected, inputs)


@pytest.mark.parametrize("entry", ENTRIES, ids=[e["key"] for e in ENTRIES])
def test_tensor_strided_schedule_matches_reference_golden(entry):
    # the default (contiguous, pieces merged in-kernel) is covered above; whole items, strided, here
    case, seed, dtype, causal, pattern = entry_params(entry)
    inputs = build_case(case, seed, dtype, causal, pattern)
    expected = dtype_bits_to_f32(expected_bits(entry), dtype_name(dtype))
    _check(_run(inputs, path="tensor", task_assignment="strided"), expected, inputs)


@pytest.mark.parametrize("kernel", ["auto", "halves"])
@pytest.mark.parametrize("schedule,causal,programs",
                         [("contiguous", False, 1), ("contiguous", False, 3), ("contiguous", False, 7),
                          ("contiguous", False, None), ("contiguous", True, 28), ("contiguous", True, None),
                          ("tail", False, 1), ("tail", False, 4), ("tail", False, 5), ("tail", False, 7),
                          ("tail", False, None), ("tail", True, 28)])
def test_contiguous_schedule_pieces_merge_to_the_oracle(schedule, causal, programs, kernel):
    # Few programs over many KV tiles: items are cut into pieces at arbitrary tile offsets, some items
    # span many programs, and the last arriver of each merges them in the same launch. (The reference's
    # general route, taken when causal, accepts only its default program caps.)
    case = ("stream_pieces", 3, 600, 2, 128, 128, 20)  # B3 Sq600 (3 query pairs) H2 D128 page 128
    from fixtures import make_inputs, poison_unread
    q, k, v, table = make_inputs(case, 42, torch.bfloat16)
    lengths = [2560, 1, 1333]
    k, v = poison_unread(k, v, table, lengths, 128)
    inputs = {"case": case, "seed": 42, "dtype": torch.bfloat16, "causal": causal, "pattern": "stream", "q": q,
              "k": k, "v": v, "table": table, "lengths": torch.tensor(lengths, dtype=torch.int32)}
    # 18 items (3 requests x 2 heads x 3 query pairs): the tail schedule deals floor(18 / G) * G whole items
    # strided and cuts only the rest (none with one program, all of them with 148)
    kwargs = dict(path="tensor", task_assignment=schedule, tensor_kernel=kernel)
    if programs is not None:
        kwargs["persistent_programs"] = programs
    out = _run(inputs, **kwargs)
    _check(out, oracle_output(inputs), inputs)
    # twice in a row: the arrival counters are reset for the next launch
    out2 = _run(inputs, **kwargs)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("schedule,causal,programs,dim,sq", [
    ("contiguous", False, 1, 128, 1), ("contiguous", False, 3, 128, 1), ("contiguous", False, 7, 64, 3),
    ("contiguous", True, 5, 128, 8), ("contiguous", False, None, 256, 2), ("contiguous", True, None, 128, 4),
    ("tail", False, 5, 128, 1), ("tail", True, 7, 64, 8), ("tail", False, None, 128, 1),
    ("strided", False, None, 128, 1), ("strided", True, 3, 256, 5)])
def test_decode_contiguous_schedule_pieces_merge_to_the_oracle(schedule, causal, programs, dim, sq):
    # Decode kernel, one split: the KV stages of all (request, query-row block, head) items are cut into equal
    # ranges per program, so long requests are cut into pieces held by several CTAs and merged in place by the
    # one completing the set; empty and short requests cost one unit. Few programs force many cuts.
    case = ("decode_pieces", 4, sq, 3, dim, 64, 64)  # B4 H3, page 64, up to 4096 tokens
    from fixtures import make_inputs, poison_unread
    q, k, v, table = make_inputs(case, 7, torch.bfloat16)
    lengths = [4000, 0, 1, 777]
    k, v = poison_unread(k, v, table, lengths, 64)
    inputs = {"case": case, "seed": 7, "dtype": torch.bfloat16, "causal": causal, "pattern": "decode_pieces",
              "q": q, "k": k, "v": v, "table": table, "lengths": torch.tensor(lengths, dtype=torch.int32)}
    from fgw_b200.operators.mha.current import build_kernel
    dev = torch.device("cuda", 0)
    args = [inputs[key].to(dev) for key in ("q", "k", "v", "table", "lengths")]
    kwargs = dict(path="decode", task_assignment=schedule, _b200_splits=1)  # one split (page 64: fallback route)
    if programs is not None:
        kwargs["persistent_programs"] = programs
    kernel = build_kernel(4, sq, 3, dim, k.shape[0], 64, 64, causal, "bfloat16", 0, **kwargs)
    assert kernel.num_splits == 1 and kernel.task_assignment == schedule
    out = kernel(*args)
    torch.cuda.synchronize()
    _check(out, oracle_output(inputs), inputs)
    out2 = kernel(*args)  # the arrival counters are reset for the next launch
    torch.cuda.synchronize()
    assert torch.equal(out, out2)


SPLIT_ENTRIES = [e for e in ENTRIES if e["seed"] == 7 and e["pattern"] == "mixed"]


@pytest.mark.parametrize("kernel", ["auto", "halves"])
@pytest.mark.parametrize("splits", [2, 8])
@pytest.mark.parametrize("entry", SPLIT_ENTRIES, ids=[e["key"] for e in SPLIT_ENTRIES])
def test_tensor_path_splits_match_oracle(entry, splits, kernel):
    case, seed, dtype, causal, pattern = entry_params(entry)
    if splits > (case[5] * case[6] + 31) // 32:
        pytest.skip("more splits than 32-token tiles in table capacity")
    if kernel == "halves" and case[4] > 128:
        pytest.skip("the key-halves kernel serves head dims up to 128")
    inputs = build_case(case, seed, dtype, causal, pattern)
    _check(_run(inputs, path="tensor", cube_mode="general", num_splits=splits, tensor_kernel=kernel),
           oracle_output(inputs), inputs)


@pytest.mark.parametrize("kernel", ["auto", "halves"])
@pytest.mark.parametrize("dim", [16, 48, 64, 80, 128, 144, 192, 256])
@pytest.mark.parametrize("page", [16, 48, 64])
def test_tensor_path_long_causal_tails(dim, page, kernel):
    if kernel == "halves" and dim > 128:
        pytest.skip("the key-halves kernel serves head dims up to 128")
    # Config-4 style: several 128-row query tiles, causal, ragged lengths incl. 0 and partial pages,
    # 1% of K rows scaled x8 to stress the running max.
    case = (f"edge_d{dim}_p{page}", 3, 200, 2, dim, page, (700 + page - 1) // page)
    from fixtures import make_inputs, poison_unread
    q, k, v, table = make_inputs(case, 2026, torch.float16)
    lengths = [0, 699, 333]
    gen = torch.Generator().manual_seed(11)
    rows = torch.randperm(k.shape[0], generator=gen)[: max(1, k.shape[0] // 100)]
    k = k.clone()
    k[rows] = (k[rows].float() * 8).to(k.dtype)
    k, v = poison_unread(k, v, table, lengths, page)
    inputs = {"case": case, "seed": 2026, "dtype": torch.float16, "causal": True, "pattern": "edge", "q": q,
              "k": k, "v": v, "table": table, "lengths": torch.tensor(lengths, dtype=torch.int32)}
    _check(_run(inputs, path="tensor", tensor_kernel=kernel), oracle_output(inputs), inputs)


@pytest.mark.parametrize("case,splits,causal,pattern,dtype,programs", [
    (("merge_d128", 4, 1, 8, 128, 64, 40), 4, False, "mixed", torch.bfloat16, None),
    (("merge_rows", 3, 5, 4, 128, 16, 100), 16, True, "mixed", torch.bfloat16, None),
    (("merge_d64", 8, 2, 16, 64, 128, 12), 2, False, "full", torch.float16, None),
    (("merge_d256", 2, 1, 2, 256, 64, 24), 8, True, "mixed", torch.bfloat16, None),
    (("merge_groups", 64, 1, 32, 128, 64, 16), 4, False, "mixed", torch.float16, None),
    # 3 heads on 3 programs: every split of a row group is an item of the same CTA, which counts itself in
    # once per split and merges on the last; and one program doing everything
    (("merge_one_cta", 2, 1, 3, 128, 128, 16), 8, False, "mixed", torch.bfloat16, 3),
    (("merge_one_program", 3, 1, 2, 128, 128, 8), 4, True, "full", torch.bfloat16, 1),
], ids=lambda v: v[0] if isinstance(v, tuple) else None)
def test_decode_split_merge_in_place_matches_the_merge_launch(case, splits, causal, pattern, dtype, programs):
    # fgw_mha_paged_fwd merges the decode kernel's splits in place: the CTA whose arrival completes a row
    # group's split set merges it. fgw_mha_partial + fgw_mha_merge do the same merge in a second launch with
    # the same arithmetic, so the two outputs are the same bits; a second call on the same workspace (arrival
    # counters zeroed again by the plan kernel) gives them again. Cases include splits past a request's
    # KV tiles (empty partials) and empty requests.
    from fgw_b200.operators.mha.current import build_kernel
    dev = torch.device("cuda", 0)
    inputs = build_case(case, 7, dtype, causal, pattern)
    args = [inputs[key].to(dev) for key in ("q", "k", "v", "table", "lengths")]
    # the general route takes only its default program cap; the BF16 D128 page-128 route takes any cap
    extra = dict(cube_mode="general") if programs is None else dict(persistent_programs=programs)
    kernel = build_kernel(case[1], case[2], case[3], case[4], args[1].shape[0], case[6], case[5], causal,
                          dtype_name(dtype), 0, num_splits=splits, path="decode", **extra)
    assert kernel.num_splits == splits
    if programs is not None:
        assert kernel.compute_grid == programs
    ws = kernel.new_workspace(dev)
    fused = kernel(*args, workspace=ws).clone()
    again = kernel(*args, workspace=ws)
    separate_ws = kernel.new_workspace(dev)
    kernel.partial_kernel(*args, separate_ws)
    separate = kernel.merge_kernel(*args, separate_ws)
    torch.cuda.synchronize()
    assert torch.equal(fused.view(torch.int16), separate.view(torch.int16))
    assert torch.equal(again.view(torch.int16), fused.view(torch.int16))
    _check(fused, oracle_output(inputs), inputs)


@pytest.mark.parametrize("splits,dtype", [(64, torch.bfloat16), (128, torch.float16)])
def test_b200_split_counts_beyond_the_reference_set(splits, dtype):
    # The B200 split model may pick 64 or 128 splits (one request and head over a long cache fills only
    # `splits` SMs); an explicit num_splits keeps the reference's accepted set. Long ragged caches, many
    # empty splits for the short request; in-place merge against the merge launch and the oracle.
    from fgw_b200.operators.mha.current import build_kernel
    case = ("many_splits", 2, 1, 2, 128, 128, 160)  # table capacity 20480 tokens = 160 KV tiles
    dev = torch.device("cuda", 0)
    inputs = build_case(case, 42, dtype, False, "mixed")
    args = [inputs[key].to(dev) for key in ("q", "k", "v", "table", "lengths")]
    shape = (case[1], case[2], case[3], case[4], args[1].shape[0], case[6], case[5], False, dtype_name(dtype), 0)
    with pytest.raises(ValueError):
        build_kernel(*shape, cube_mode="general", num_splits=splits)
    for bad in (dict(_b200_splits=3), dict(_b200_splits=256), dict(_b200_splits=splits, num_splits=2)):
        with pytest.raises(ValueError):  # not a candidate / past the 160 KV tiles / both ways at once
            build_kernel(*shape, **bad)
    kernel = build_kernel(*shape, _b200_splits=splits, path="decode")
    assert kernel.num_splits == splits
    fused = kernel(*args)
    separate_ws = kernel.new_workspace(dev)
    kernel.partial_kernel(*args, separate_ws)
    separate = kernel.merge_kernel(*args, separate_ws)
    torch.cuda.synchronize()
    assert torch.equal(fused.view(torch.int16), separate.view(torch.int16))
    _check(fused, oracle_output(inputs), inputs)
