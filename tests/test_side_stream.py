"""Selection sorts run on a side stream from the program's start, alongside
the forward kernels.  The lowering must keep every buffer a side kernel
touches (its scratch included) allocated until the main stream joins the side
stream; it checks that invariant, and that no two live buffers share bytes,
when it places the arena (a violation fails the compile).  These tests lower
plans with a scatter-add on the host and read the join point back."""
import re

import pytest

from poorgrad_b200 import backend, configs


@pytest.mark.parametrize("name,kw", [("charmlp", {}), ("charmlp", dict(batch=64, hidden=32, embed=8)),
                                     ("gpt2", dict(layers=1, seq=64, batch=2, vocab=97, d=32, heads=2, mlp=64))])
def test_sorts_lead_and_join_before_their_consumers(built, name, kw):
    try:
        w = configs.BUILDERS[name](**kw)
    except TypeError:
        pytest.skip("config does not take these sizes")
    text = backend.lower_describe(w.columns)
    lines = text.splitlines()
    kernels = [l for l in lines if re.match(r"\d+: ", l)]
    sorts = [i for i, l in enumerate(kernels) if " sort selection" in l]
    assert sorts and sorts == list(range(len(sorts))), "sorts are not at the front"
    join = int(re.search(r"^side join (\d+)$", text, re.M).group(1))
    first_consumer = min(i for i, l in enumerate(kernels) if ": scatter " in l)
    assert len(sorts) <= join <= first_consumer
