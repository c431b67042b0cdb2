"""Host logic of adjust_logits (sampling/compact.py:14-79 of the reference): the steps are
gathered into as few dsv_adjust_logits passes as their order allows (a pass applies additive,
scaling, mask, bias in that order), and every penalizer stage of the orchestrator keeps a pass
of its own.  No GPU: the launches are recorded."""

from dspine_b200.sampling.compact import _Plan


def _record(steps):
    calls = []
    plan = _Plan(lambda **kw: calls.append(sorted(kw)))
    for step in steps:
        plan.add(*step)
    plan.flush()
    return calls


def test_usual_batch_is_one_pass():
    assert _record([("additive", 1), ("scaling", 2), ("bitmask", 3), ("bias", 4)]) == [
        ["additive", "bias", "bitmask", "scaling"]]


def test_absent_steps_launch_nothing():
    assert _record([("additive", None), ("bias", None)]) == []


def test_penalizer_stages_open_their_own_passes():
    calls = _record([("additive", 1), ("scaling", 2), ("additive", 5, True), ("scaling", 6, True),
                     ("bitmask", 3), ("bias", 4)])
    assert calls == [["additive", "scaling"], ["additive"], ["bias", "bitmask", "scaling"]]


def test_out_of_order_step_starts_a_new_pass():
    assert _record([("bias", 4), ("additive", 1)]) == [["bias"], ["additive"]]
