"""Reasoning controls (reference src/engine/reasoning_controls.rs): overthinking from
next-token distributions, repetition, termination policies, chains and statistics."""
import math

import pytest
import torch

from lightbulb_b200.extras.reasoning import (DecodingBudget, OverthinkingDetector,
                                             ReasoningController, TerminationPolicy,
                                             logits_stats)


def _peaked(v=64, top=0, margin=20.0):
    x = torch.zeros(v)
    x[top] = margin
    return x


def test_logits_stats_matches_definition():
    x = torch.randn(3, 50)
    e, p = logits_stats(x)
    pr = torch.softmax(x, -1)
    assert torch.allclose(e, -(pr * pr.log()).sum(-1), atol=1e-5)
    assert torch.allclose(p, pr.max(-1).values)
    e2, p2 = logits_stats(torch.zeros(1, 8))          # uniform: ln 8, 1/8
    assert abs(e2.item() - math.log(8)) < 1e-5 and abs(p2.item() - 0.125) < 1e-6


def test_overthinking_needs_low_entropy_and_low_variance():
    d = OverthinkingDetector(window_size=5)
    assert not d.is_overthinking_logits([_peaked()] * 4)          # window not filled
    assert d.is_overthinking_logits([_peaked()] * 5)              # confident and stable
    assert not d.is_overthinking_logits([torch.zeros(64)] * 5)    # high entropy
    # alternating confident / unconfident: top-prob variance above 0.1
    flip = [_peaked() if i % 2 else torch.zeros(64) for i in range(5)]
    assert not d.is_overthinking_logits(flip)
    assert not OverthinkingDetector(enabled=False).is_overthinking_logits([_peaked()] * 5)


def test_repetition():
    d = OverthinkingDetector(window_size=3)
    assert d.is_repeating([9, 1, 2, 3, 1, 2, 3])
    assert not d.is_repeating([1, 2, 3, 1, 2, 4])
    assert not d.is_repeating([1, 2, 3, 1, 2])


def test_termination_policies():
    assert TerminationPolicy.fixed_steps(3).should_terminate(3, 0.0, [], 0)
    assert not TerminationPolicy.fixed_steps(3).should_terminate(2, 0.0, [], 0)
    assert TerminationPolicy.confidence(0.9).should_terminate(1, 0.95, [], 0)
    conv = TerminationPolicy.convergence(3, 0.01)
    assert not conv.should_terminate(1, 0, [0.5, 0.5], 0)
    assert conv.should_terminate(1, 0, [0.1, 0.5, 0.5, 0.51], 0)
    assert TerminationPolicy.special_token(7).should_terminate(1, 0, [], 7)
    both = TerminationPolicy.combined([TerminationPolicy.special_token(7),
                                       TerminationPolicy.confidence(0.99)])
    assert both.should_terminate(1, 0.995, [], 1) and not both.should_terminate(1, 0.5, [], 1)


def test_controller_order_budget_and_stats():
    c = ReasoningController(DecodingBudget(max_chains=2, max_steps_per_chain=4,
                                           max_total_tokens=100),
                            OverthinkingDetector(window_size=3),
                            TerminationPolicy.special_token(99))
    a = c.start_chain()
    assert not c.record_step(a, 5, 0.4, stats=(2.0, 0.3))
    assert not c.record_step(a, 6, 0.5, stats=(2.0, 0.4))
    assert c.record_step(a, 99, 0.6, stats=(2.0, 0.5))             # special token
    assert c.get_chain(a).termination_reason == "Termination policy triggered"
    b = c.start_chain()
    with pytest.raises(RuntimeError):
        c.start_chain()                                             # max chains
    for t in range(3):
        stop = c.record_step(b, t, 0.9, logits=_peaked())
    assert stop and c.get_chain(b).termination_reason == "Overthinking detected"
    st = c.stats()
    assert st.total_chains == 2 and st.completed_chains == 2 and st.total_tokens == 6
    assert abs(st.avg_steps_per_chain - 3.0) < 1e-9
    c.reset()
    assert c.stats().total_chains == 0


def test_controller_step_and_token_budgets():
    c = ReasoningController(DecodingBudget(max_steps_per_chain=2, max_total_tokens=3),
                            OverthinkingDetector(enabled=False),
                            TerminationPolicy.fixed_steps(100))
    x = c.start_chain()
    assert not c.record_step(x, 1, 0.1) and not c.record_step(x, 2, 0.1)
    assert c.record_step(x, 3, 0.1)
    assert c.get_chain(x).termination_reason == "Budget: max steps reached"
    y = c.start_chain()
    assert not c.record_step(y, 1, 0.1)
    assert c.record_step(y, 2, 0.1)
    assert c.get_chain(y).termination_reason == "Budget: max tokens reached"
