"""Draft-depth controller of speculative serving (CPU): more acceptance or a
cheaper drafter deepens the tree; the break-even acceptance matches the cost
model."""
from swarmllm_b200.engine.spec_engine import SpecController


def test_depth_follows_acceptance_and_costs():
    c = SpecController(max_depth=6)
    assert c.best_depth() == 6                      # no measurement yet: the configured depth
    for _ in range(30):
        c.observe(4, 3.8, t_draft=4 * 0.001, t_verify=0.010)   # nearly everything accepted
    deep = c.best_depth()
    assert deep >= 5
    for _ in range(60):
        c.observe(4, 0.1, t_draft=4 * 0.004, t_verify=0.010)   # drafts rejected, drafter slow
    assert c.best_depth() < deep and c.best_depth() <= 2


def test_break_even_acceptance():
    c = SpecController(max_depth=4)
    c.observe(4, 2.0, t_draft=4 * 0.002, t_verify=0.010)
    a = c.break_even_accept(4)
    # at the break-even rate a round commits as many tokens as its cost in verify units
    cost = (c.t_draft * 4 + c.t_verify) / c.t_verify
    assert abs(sum(a ** i for i in range(5)) - cost) < 1e-6
    assert 0.0 < a < 1.0
