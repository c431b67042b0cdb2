"""dsv_verify_logits_noalloc: the same verification with the library's fixed device scratch.

This entry point has no counterpart in the reference; it serves callers that cannot allocate
device memory at verification time.  It must give exactly what dsv_verify_logits gives on the
same inputs, on two calls in a row (the scratch it reuses is cleared by each call), for every
dtype path, with and without the accept-compact outputs.  The file's name puts it last in the
collection order, so it also runs after every other GPU test has used the library.
"""

import pytest
import torch

from dspine_b200 import verify, workloads

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _batch(seed, B, V, dtype):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, 17, (B,), generator=g, dtype=torch.int32)
    temperature = torch.rand(B, generator=g) * 1.5
    temperature[torch.rand(B, generator=g) < 0.25] = 0.0
    ks = torch.tensor([workloads.TOPK_OFF, 1, 20, 50], dtype=torch.int32)
    top_k = ks[torch.randint(0, len(ks), (B,), generator=g)]
    top_p = 0.8 + 0.2 * torch.rand(B, generator=g)
    b = workloads.build(lens, temperature, top_k, top_p, V=V, dtype=dtype, seed=seed)
    return b.to(DEV)


def _same(a, b):
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("dtype,V,B", [(torch.bfloat16, 151936, 64), (torch.bfloat16, 4099, 256),
                                       (torch.float32, 4099, 32)])
def test_noalloc_matches_workspace_entry_point(dtype, V, B):
    batch = _batch(7 + B, B, V, dtype)
    kw = batch.kwargs()
    comp_ref = verify.CompactOutputs.allocate(B, DEV)
    ref = verify.verify_logits(**kw, outputs=verify.new_outputs(B, DEV), slots=batch.slots,
                               slot_rows=batch.slot_rows, compact=comp_ref,
                               workspace=verify.workspace_for(B, DEV))
    torch.cuda.synchronize()
    assert verify.workspace_for(B, DEV).error_word() == 0
    for call in range(2):  # two calls in a row reuse the same scratch
        out = verify.new_outputs(B, DEV)
        for o in out:
            o.fill_(-7)
        comp = verify.CompactOutputs.allocate(B, DEV)
        err = torch.full((1,), -1, dtype=torch.int32, device=DEV)
        verify.verify_logits_noalloc(**kw, outputs=out, slots=batch.slots,
                                     slot_rows=batch.slot_rows, compact=comp, device_error=err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0, f"call {call}: device error word {int(err.item()):#x}"
        _same(out, ref)
        n = int(comp_ref.offsets[-1].item())
        assert int(comp.offsets[-1].item()) == n
        assert torch.equal(comp.offsets, comp_ref.offsets)
        assert torch.equal(comp.tokens[:n], comp_ref.tokens[:n])
        assert torch.equal(comp.kept_slots[:n], comp_ref.kept_slots[:n])
        assert torch.equal(comp.freed_offsets, comp_ref.freed_offsets)
        m = int(comp_ref.freed_offsets[-1].item())
        assert torch.equal(comp.freed_slots[:m], comp_ref.freed_slots[:m])


def test_noalloc_without_compact_or_error_word():
    batch = _batch(3, 16, 4099, torch.bfloat16)
    kw = batch.kwargs()
    ref = verify.verify_logits(**kw, outputs=verify.new_outputs(16, DEV))
    for _ in range(2):
        out = verify.verify_logits_noalloc(**kw, outputs=verify.new_outputs(16, DEV))
        torch.cuda.synchronize()
        _same(out, ref)


def test_noalloc_rejects_batches_beyond_its_scratch():
    from dspine_b200 import _lib
    batch = _batch(5, 257, 97, torch.bfloat16)
    with pytest.raises(ValueError):
        verify.verify_logits_noalloc(**batch.kwargs(), outputs=verify.new_outputs(257, DEV))
    # the C ABI refuses it too (status 6: scratch too small), before enqueuing anything
    st = _lib.load().dsv_verify_logits_noalloc(257, 97, 0, *([None] * 3), 1, *([None] * 2), 0,
                                               97, *([None] * 12), None, None, None)
    assert st == 6
