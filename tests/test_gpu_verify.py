"""Parity of the fused CUDA verification (dsv_verify_logits) with the CPU oracle.

Every case compares all five outputs (accept, commit, bonus, output, new_seq) bit-exactly:
the kernel and the oracle use the same exact fixed-point sums, so no tolerance applies to
these integer outputs.  Cases follow the reference's own parity tests
(tests/test_sparse_accept_compact.py:56-130, tests/test_dynamic_sampling.py:222-338): ragged
caps, all-accepted rows, zero-residual fallback, greedy ties, mixed filters.
"""

import numpy as np
import pytest
import torch

import oracle as O
from dspine_b200 import verify, workloads
from tests.helpers import assert_same, oracle_verify

pytestmark = pytest.mark.gpu

DEV = "cuda"


def run_kernel(batch, compact=False):
    kw = batch.kwargs()
    out = verify.verify_logits(**kw)
    torch.cuda.synchronize()
    # no bulk-copy timeout, bad row, bad slot or (index-checking builds) failed index check
    assert verify.workspace_for(batch.B, DEV).error_word() == 0
    return out


def random_batch(seed, B, V, dtype, quantize=False, with_draft=True, neg_inf=False):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, 17, (B,), generator=g, dtype=torch.int32)
    lens[0] = 16
    temperature = torch.rand(B, generator=g) * 1.8
    temperature[torch.rand(B, generator=g) < 0.2] = 0.0
    ks = torch.tensor([workloads.TOPK_OFF, 1, 3, 7, 20, 50], dtype=torch.int32)
    top_k = ks[torch.randint(0, len(ks), (B,), generator=g)]
    top_p = torch.where(torch.rand(B, generator=g) < 0.3, torch.ones(B),
                        0.5 + 0.5 * torch.rand(B, generator=g))
    batch = workloads.build(lens, temperature, top_k, top_p, V=V, dtype=torch.float32,
                            seed=seed, with_draft=with_draft)
    if quantize:  # many exactly equal logits: ties at every boundary
        batch.target_logits = (batch.target_logits * 2).round() / 2
        if batch.draft_logits is not None:
            batch.draft_logits = (batch.draft_logits * 2).round() / 2
    if neg_inf:
        batch.target_logits[:, ::5] = -float("inf")
    batch.uniforms[0] = 0.0  # request 0: everything accepted when q agrees
    batch.target_logits = batch.target_logits.to(dtype)
    if batch.draft_logits is not None:
        batch.draft_logits = batch.draft_logits.to(dtype)
    return batch.to(DEV)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("V", [97, 257, 1031, 4099])
def test_small_vocab_matches_oracle(dtype, V):
    for seed in range(3):
        batch = random_batch(1000 + seed * 7 + V, 9, V, dtype)
        got = run_kernel(batch)
        assert_same(got, oracle_verify(batch), f"V={V} seed={seed}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_ties_and_masked_logits(dtype):
    for seed in range(3):
        batch = random_batch(77 + seed, 12, 2053, dtype, quantize=True, neg_inf=seed == 1)
        assert_same(run_kernel(batch), oracle_verify(batch), f"ties seed={seed}")


@pytest.mark.parametrize("V", [4099, 151936])
def test_every_selection_path(V):
    """Rows that resolve in the top window, rows whose nucleus needs the histogram levels,
    top_k beyond the window, a window overflow (all-equal logits) and unfiltered rows."""
    off = workloads.TOPK_OFF
    params = [  # (temperature, top_k, top_p)
        (1.5, off, 0.95), (0.3, off, 0.9), (1.0, 500, 1.0), (1.0, 500, 0.5),
        (1.0, 192, 0.99), (0.7, 20, 0.3), (1.0, 20, 0.9), (1.0, off, 1.0),
        (2.0, off, 0.999), (0.05, off, 0.8), (1.2, 7, 1.0), (0.9, 50, 0.85),
    ]
    B = len(params)
    g = torch.Generator().manual_seed(V)
    lens = torch.randint(2, 17, (B,), generator=g, dtype=torch.int32)
    temperature, top_k, top_p = (torch.tensor(x) for x in zip(*params))
    batch = workloads.build(lens, temperature.float(), top_k.int(), top_p.float(), V=V,
                            dtype=torch.float32, seed=V + 1)
    # request 6: every logit equal -> every element enters the top window (overflow path)
    b = 6
    t0, n = int(batch.target_rows[b]), int(lens[b])
    batch.target_logits[t0:t0 + n] = 1.0
    d0 = int(batch.draft_rows[b])
    batch.draft_logits[d0:d0 + n - 1] = 1.0
    batch.target_logits = batch.target_logits.to(torch.bfloat16)
    batch.draft_logits = batch.draft_logits.to(torch.bfloat16)
    batch = batch.to(DEV)
    assert_same(run_kernel(batch), oracle_verify(batch), f"paths V={V}")
    assert verify.workspace_for(batch.B, DEV).error_word() == 0


def test_one_hot_q_without_draft_logits():
    batch = random_batch(5, 17, 1031, torch.bfloat16, with_draft=False)
    assert batch.draft_logits is None
    assert_same(run_kernel(batch), oracle_verify(batch), "one-hot q")


def test_zero_residual_falls_back_to_target():
    """tests/test_sparse_accept_compact.py:77-86: p == q on the rejected row."""
    batch = random_batch(9, 4, 257, torch.float32)
    # draft == target for request 1 and a coin that rejects (u = 1 -> u*q < p fails)
    b = 1
    t0, d0 = int(batch.target_rows[b]), int(batch.draft_rows[b])
    n = int(batch.verify_lens[b]) - 1
    if n > 0:
        batch.draft_logits[d0:d0 + n] = batch.target_logits[t0:t0 + n]
    batch.uniforms[b] = 1.0
    assert_same(run_kernel(batch), oracle_verify(batch), "zero residual")


def test_repeated_launches_are_identical_and_reset_the_workspace():
    batch = random_batch(31, 23, 4099, torch.bfloat16)
    first = [t.clone() for t in run_kernel(batch)]
    for _ in range(3):
        again = run_kernel(batch)
        for a, b in zip(first, again):
            assert torch.equal(a, b)
    ws = verify.workspace_for(batch.B, DEV)
    assert ws.error_word() == 0
    header = ws.buf[:16].view(torch.int32).cpu().tolist()
    assert header[:3] == [0, 0, 0]


def test_config0_full_vocab_fp32():
    batch = workloads.config0(device=DEV)
    assert_same(run_kernel(batch), oracle_verify(batch), "config0")


def test_config1_full_size_bf16():
    batch = workloads.config1(device=DEV)
    assert_same(run_kernel(batch), oracle_verify(batch), "config1")


def test_config4_full_size_bf16():
    batch = workloads.config4(device=DEV)
    assert_same(run_kernel(batch), oracle_verify(batch), "config4")


def test_accept_compact_matches_oracle():
    batch = workloads.config1(device=DEV, B=64, V=4099)
    comp = verify.CompactOutputs.allocate(batch.B, DEV)
    out = verify.verify_logits(**batch.kwargs(), slots=batch.slots, slot_rows=batch.slot_rows,
                               compact=comp)
    torch.cuda.synchronize()
    acc, commit, bonus, output, new_seq = [t.cpu().numpy() for t in out]
    tok, sl, off, fr, foff = O.accept_compact(commit, batch.verify_lens.cpu().numpy(), output,
                                              batch.slots.cpu().numpy(),
                                              batch.slot_rows.cpu().numpy())
    n, nf = int(off[-1]), int(foff[-1])
    np.testing.assert_array_equal(comp.offsets.cpu().numpy(), off)
    np.testing.assert_array_equal(comp.freed_offsets.cpu().numpy(), foff)
    np.testing.assert_array_equal(comp.tokens[:n].cpu().numpy(), tok)
    np.testing.assert_array_equal(comp.kept_slots[:n].cpu().numpy(), sl)
    np.testing.assert_array_equal(comp.freed_slots[:nf].cpu().numpy(), fr)
    assert verify.workspace_for(batch.B, DEV).error_word() == 0


def test_invalid_arguments_raise_before_launch():
    batch = random_batch(3, 4, 257, torch.bfloat16)
    kw = batch.kwargs()
    with pytest.raises(ValueError):
        verify.verify_logits(**{**kw, "candidates": kw["candidates"][:, :15]})
    with pytest.raises(ValueError):
        verify.verify_logits(**{**kw, "top_k": kw["top_k"].long()})
    with pytest.raises(ValueError):
        verify.verify_logits(**{**kw, "draft_logits": kw["draft_logits"].float()})


@pytest.mark.parametrize("case", ["plain", "ties", "outside", "band", "inf"])
def test_split_rows_match_oracle(case):
    """More selection rows than CTAs of the row kernel: the rows beyond the first wave are
    split in two halves whose histograms meet through the workspace.  Every request sampled
    with top_p < 1 and 16 positions, so 64 requests give 1984 one-pass rows; the cases put
    ties, values outside the fixed histogram range (the halves fall back to the full-row path),
    values in the listed band, and -inf into those rows."""
    g = torch.Generator().manual_seed({"plain": 1, "ties": 2, "outside": 3, "band": 4, "inf": 5}[case])
    B, V = 64, 4096
    lens = torch.full((B,), 16, dtype=torch.int32)
    temperature = 0.3 + torch.rand(B, generator=g)
    top_k = torch.where(torch.rand(B, generator=g) < 0.5, torch.tensor(workloads.TOPK_OFF),
                        torch.tensor(50)).to(torch.int32)
    top_p = 0.6 + 0.39 * torch.rand(B, generator=g)
    batch = workloads.build(lens, temperature, top_k, top_p, V=V, dtype=torch.float32, seed=5)
    t, d = batch.target_logits, batch.draft_logits
    if case == "ties":
        t.copy_((t * 2).round() / 2)
        d.copy_((d * 2).round() / 2)
    elif case == "outside":
        t[1::3, 7] = 5000.0  # above the fixed range in some rows, in one half or the other
        t[2::3, 3000] = -6000.0
    elif case == "band":
        t[:, 100:140] = 1e-7  # |v| < 2^-20: listed element by element
        d[:, 2100:2130] = -3e-8
    elif case == "inf":
        t[:, ::7] = -float("inf")
    batch.target_logits = t.to(torch.bfloat16)
    batch.draft_logits = d.to(torch.bfloat16)
    batch = batch.to(DEV)
    assert_same(run_kernel(batch), oracle_verify(batch), f"split rows {case}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", ["accept", "reject", "mixed"])
def test_dropped_rows_do_not_change_outputs(case, dtype):
    """A chain stops at its first rejected step, so the row kernel drops (at dequeue, or during
    a row's first pass) the rows after a known rejection and the rows of a request whose outcome
    is known.  Drafts equal to the target accept every step (no row can be dropped), drafts
    opposite to it reject at once (most rows are dropped); outputs equal the oracle's, which
    processes every row, and the bytes read show what was dropped.  fp32 logits take the
    cluster kernel, which drops whole (request, position) tasks past a known rejection."""
    g = torch.Generator().manual_seed(77)
    B, V = 64, 4099
    lens = torch.full((B,), 16, dtype=torch.int32)
    lens[::5] = torch.randint(1, 16, (len(lens[::5]),), generator=g, dtype=torch.int32)
    temperature = 0.4 + torch.rand(B, generator=g)
    temperature[::7] = 0.0
    top_k = torch.where(torch.rand(B, generator=g) < 0.5, torch.tensor(workloads.TOPK_OFF),
                        torch.tensor(20)).to(torch.int32)
    top_p = 0.7 + 0.3 * torch.rand(B, generator=g)
    batch = workloads.build(lens, temperature, top_k, top_p, V=V, dtype=torch.float32, seed=9)
    batch.target_logits = batch.target_logits.to(dtype)
    batch.draft_logits = batch.draft_logits.to(dtype)
    if case == "accept":
        # draft row (b, s) is target row (b, s), so q = p; drafted tokens are each row's first
        # argmax (kept by every filter; what greedy requests accept)
        batch.draft_logits = batch.target_logits.clone()
        batch.draft_rows = batch.target_rows.clone()
        am = batch.target_logits.float().argmax(dim=1)
        rows = batch.target_rows.long()
        for b in range(B):
            n = int(lens[b])
            batch.candidates[b, 1:n] = am[rows[b]:rows[b] + n - 1]
    elif case == "reject":
        batch.draft_logits = -batch.draft_logits
    batch = batch.to(DEV)
    ws = verify.workspace_for(batch.B, DEV)
    ws.prepare(batch.B)  # a change of batch size zeroes the workspace (and its byte counter)
    before = ws.bytes_read()
    got = run_kernel(batch)
    read = ws.bytes_read() - before
    expected = oracle_verify(batch)
    assert_same(got, expected, f"dropped rows {case} {dtype}")
    all_rows = batch.algorithmic_bytes()
    if case == "accept":
        assert (expected[0] == batch.verify_lens.cpu().numpy() - 1).all()
        assert read >= all_rows  # every row read (16-byte vectors round each row up)
    elif case == "reject":
        assert read < all_rows // 2


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("case", ["random", "accept", "config1"])
def test_host_inputs_copy_only_what_the_outcome_needs(case, dtype):
    """verify_logits_host on CPU (pinned) inputs: rows copied in widening windows of verify
    positions, each window verified with lengths capped at it; outputs and compaction equal the
    device call on the whole batch (and the oracle), and fewer logit bytes cross to the device
    unless every step is accepted."""
    if case == "config1":
        if dtype == torch.float32:
            pytest.skip("config 1 is bf16")
        batch = workloads.config1()
    else:
        batch = random_batch(4242, 48, 4099, dtype).to("cpu")
        if case == "accept":
            batch.draft_logits = batch.target_logits.clone()
            batch.draft_rows = batch.target_rows.clone()
            am = batch.target_logits.float().argmax(dim=1)
            for b in range(batch.B):
                n = int(batch.verify_lens[b])
                r0 = int(batch.target_rows[b])
                batch.candidates[b, 1:n] = am[r0:r0 + n - 1]
    kw = {k: v.pin_memory() for k, v in batch.kwargs().items() if v is not None}
    slots, slot_rows = batch.slots.pin_memory(), batch.slot_rows.pin_memory()
    got, comp, info = verify.verify_logits_host(**kw, slots=slots, slot_rows=slot_rows,
                                                device=DEV)
    dev_batch = batch.to(DEV)
    want_comp = verify.CompactOutputs.allocate(batch.B, DEV)
    want = verify.verify_logits(**dev_batch.kwargs(), slots=dev_batch.slots,
                                slot_rows=dev_batch.slot_rows, compact=want_comp)
    torch.cuda.synchronize()
    assert verify.workspace_for(batch.B, DEV).error_word() == 0
    for g, w in zip(got, want):
        assert torch.equal(g, w.cpu())
    n_tok = int(want[1].sum())
    assert torch.equal(comp.offsets, want_comp.offsets.cpu())
    assert torch.equal(comp.tokens[:n_tok], want_comp.tokens[:n_tok].cpu())
    assert torch.equal(comp.kept_slots[:n_tok], want_comp.kept_slots[:n_tok].cpu())
    n_free = int(want_comp.freed_offsets[-1])
    assert torch.equal(comp.freed_slots[:n_free], want_comp.freed_slots[:n_free].cpu())
    if case != "accept":
        assert_same(got, oracle_verify(batch), f"host inputs {case}")
    logit_bytes = batch.target_logits.numel() * batch.target_logits.element_size() + (
        batch.draft_logits.numel() * batch.draft_logits.element_size())
    if case == "config1":
        assert info.h2d_bytes < logit_bytes // 2
    assert info.windows[0] == 2


def test_copy_row_ranges_merges_and_copies_exactly_the_ranges():
    """dsv_copy_row_ranges: rows [first, first + n) of each range reach the device buffer at
    the same rows (adjacent ranges merged into one copy); every other row stays untouched."""
    g = torch.Generator().manual_seed(3)
    host = torch.randint(0, 1 << 15, (300, 97), generator=g, dtype=torch.int16).pin_memory()
    dev = torch.full((300, 97), -1, dtype=torch.int16, device=DEV)
    first = np.array([0, 3, 5, 40, 41, 42, 200, 299], dtype=np.int64)
    count = np.array([3, 2, 0, 1, 1, 10, 50, 1], dtype=np.int64)
    from dspine_b200 import _lib
    _lib.call("dsv_copy_row_ranges", dev.data_ptr(), host.data_ptr(), 97 * 2, len(first),
              first.ctypes.data, count.ctypes.data, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    want = torch.full((300, 97), -1, dtype=torch.int16)
    for f, n in zip(first, count):
        want[f:f + n] = host[f:f + n]
    assert torch.equal(dev.cpu(), want)


@pytest.mark.parametrize("B,V", [(1, 1031), (1024, 521), (1025, 521)])
def test_batch_limits_match_oracle(B, V):
    """One request; the largest batch of the one-launch bf16 path (1024: the task table and the
    ready list at their largest); one more request (the clustered fallback path)."""
    batch = random_batch(9000 + B, B, V, torch.bfloat16)
    assert_same(run_kernel(batch), oracle_verify(batch), f"B={B} V={V}")


def test_workspace_without_split_slots():
    """A workspace that omits the split-row slots (the last kSplitCap x (slot + flag) bytes:
    256 x 33860) is accepted and gives the same outputs; no row is split then."""
    g = torch.Generator().manual_seed(8)
    B, V = 64, 2048
    lens = torch.full((B,), 16, dtype=torch.int32)
    temperature = 0.3 + torch.rand(B, generator=g)
    top_k = torch.full((B,), workloads.TOPK_OFF, dtype=torch.int32)
    top_p = 0.6 + 0.39 * torch.rand(B, generator=g)
    batch = workloads.build(lens, temperature, top_k, top_p, V=V, dtype=torch.bfloat16,
                            seed=6).to(DEV)
    full = verify.Workspace(B, DEV)
    small = verify.Workspace(B, DEV)
    small.nbytes -= 256 * 33860
    kw = batch.kwargs()
    got_full = verify.verify_logits(**kw, workspace=full)
    got_small = verify.verify_logits(**kw, workspace=small)
    torch.cuda.synchronize()
    assert full.error_word() == 0 and small.error_word() == 0
    for a_, b_ in zip(got_full, got_small):
        assert torch.equal(a_, b_)
    assert_same(got_full, oracle_verify(batch), "split slots")


def _with_min_p(batch, seed, off_fraction=0.3):
    g = torch.Generator().manual_seed(seed)
    B = batch.B
    mp = torch.rand(B, generator=g) * 0.2
    mp[torch.rand(B, generator=g) < off_fraction] = 0.0
    mp[0] = 0.05
    return mp


@pytest.mark.parametrize("mode", [verify.SEQUENTIAL, verify.TORCH, verify.JOINT])
@pytest.mark.parametrize("dtype,V,quantize", [(torch.bfloat16, 4099, False),
                                              (torch.float32, 2053, False),
                                              (torch.bfloat16, 2053, True),
                                              (torch.bfloat16, 151936, False)])
def test_min_p_and_filter_modes_match_oracle(mode, dtype, V, quantize):
    """min-p (the floor key of "p >= min_p * max p") and the three filter modes of
    runtime/worker.py:473-508: the flashinfer backend with min-p in the batch (top-k, then top-p
    against the top-k's mass, then min-p; rows with min_p 0 included), the pytorch backend
    (joint top-k / top-p and min-p), and the joint mode, which ignores min-p."""
    for seed in range(2 if V < 100000 else 1):
        batch = random_batch(500 + seed * 13 + V + mode, 10, V, dtype, quantize=quantize)
        mp = _with_min_p(batch, seed + V)
        got = verify.verify_logits(**batch.kwargs(), min_p=mp.to(DEV), mode=mode)
        torch.cuda.synchronize()
        assert verify.workspace_for(batch.B, DEV).error_word() == 0
        want = O.verify_logits(*(t.detach().cpu().numpy() for t in (
            batch.candidates, batch.target_logits.float(), batch.target_rows,
            batch.draft_logits.float(), batch.draft_rows, batch.temperature, batch.top_k,
            batch.top_p, batch.verify_lens, batch.uniforms, batch.uniform_final,
            batch.prefix_lens)), min_p=mp.numpy(), mode=mode)
        assert_same(got, want, f"mode={mode} V={V} seed={seed}")


def test_min_p_changes_the_kept_set():
    """A min-p floor that cuts inside a top-k: the probability of a token below the floor is
    zero, so a draft of it is rejected (q > 0, p = 0) under min-p and accepted without."""
    V = 257
    logits = torch.full((2, V), -10.0)
    logits[:, 5] = 2.0
    logits[:, 9] = 0.0     # p / p_max = e^-2 = 0.135: kept at min_p 0.1, cut at 0.2
    logits[:, 11] = 1.0
    batch = workloads.build([2], [1.0], [3], [1.0], V=V, dtype=torch.float32, seed=1)
    batch.target_logits = logits[:2].clone()
    batch.draft_logits = logits[:1].clone()
    batch.candidates[0, 1] = 9
    batch.uniforms.zero_()
    batch = batch.to(DEV)
    res = {}
    for mp in (0.1, 0.2):
        got = verify.verify_logits(**batch.kwargs(), min_p=torch.tensor([mp], device=DEV),
                                   mode=verify.TORCH)
        res[mp] = int(got[0][0])
    assert res[0.1] == 1 and res[0.2] == 0
