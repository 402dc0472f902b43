"""Context planner (CPU): pinned areas, budgeted knapsack over deep history, pointers, explain."""
from fak_b200.serve.ctxplan import ContextPlanner, Layout


def _conv():
    m = [{"role": "system", "content": "You are a coding agent."}]
    for i in range(20):
        m.append({"role": "user", "content": f"step {i}: look at module_{i}.py " + "filler " * 40})
        m.append({"role": "tool", "content": f"module_{i}.py contents " + "x " * 120})
    m.append({"role": "user", "content": "now fix the bug in module_3.py please"})
    return m


def test_plan_fits_budget_and_pins_areas():
    msgs = _conv()
    p = ContextPlanner(900, layout=Layout(current_n=1, recent_n=4)).plan(msgs)
    assert p.resident_tokens <= 900 and len(p.messages) == len(msgs)
    cells = {c.index: c for c in p.cells}
    assert cells[0].area == "base" and cells[0].resident
    assert cells[len(msgs) - 1].area == "current" and cells[len(msgs) - 1].resident
    assert p.messages[-1] == msgs[-1] and p.messages[0] == msgs[0]
    # the deep cell the current turn refers to (module_3) is paged in ahead of unrelated history
    m3 = [i for i, m in enumerate(msgs) if "module_3.py contents" in m["content"]][0]
    m9 = [i for i, m in enumerate(msgs) if "module_9.py contents" in m["content"]][0]
    assert cells[m3].benefit > cells[m9].benefit and cells[m3].resident
    elided = [c for c in p.cells if not c.resident]
    assert elided and all("elided cell" in p.messages[c.index]["content"] for c in elided)


def test_large_budget_keeps_everything_exact():
    msgs = _conv()
    p = ContextPlanner(10 ** 6).plan(msgs)
    assert p.messages == msgs and all(c.resident for c in p.cells)
    assert len(p.explain()) == len(msgs)


def test_gateway_applies_the_planned_view():
    import pytest
    pytest.importorskip("fastapi")
    from fak_b200.serve import Gateway
    seen = {}

    class B:
        name, tok = "b", None

        def generate(self, ids, *a, **k):
            return iter(())

    gw = Gateway(B(), ctx_view_budget=600)
    msgs = _conv()
    view = gw._view(msgs)
    assert len(view) == len(msgs) and view != msgs and view[-1] == msgs[-1]
