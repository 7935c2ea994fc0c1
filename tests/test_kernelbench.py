"""KernelEvo Model / ModelNew contract for BASELINE's five configs.

Mirrors KernelEvo's correctness check (kernel_evo_archive/source/src/kernel_evo/core/eval/eval.py:
120-148, 525-536): the reference module is ``exec``'d for ``Model``, ``get_inputs``,
``get_init_inputs`` and the optional ``output_atol`` / ``output_rtol`` globals, the candidate
module for ``ModelNew``; outputs pass with ``torch.allclose(expected, actual, atol, rtol)``
and must be finite.
"""
import pytest
import torch

from b200fp8 import kernelbench


def _load(src):
    ns = {}
    exec(compile(src, "<task>", "exec"), ns)
    return ns


@pytest.mark.parametrize("name", sorted(kernelbench.TASKS))
def test_task_sources_define_contract(name):
    ref, new = kernelbench.task_source(name)
    r, n = _load(ref), _load(new)
    for key in ("Model", "get_inputs", "get_init_inputs", "output_atol", "output_rtol"):
        assert key in r, key
    assert "ModelNew" in n
    assert issubclass(n["ModelNew"], r["Model"])


def _flat(out):
    return list(out) if isinstance(out, (tuple, list)) else [out]


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(kernelbench.TASKS))
def test_model_new_matches_model(name):
    ref, new = kernelbench.task_source(name)
    r, n = _load(ref), _load(new)
    init = r["get_init_inputs"]()
    inputs = r["get_inputs"]()
    expected = _flat(r["Model"](*init)(*inputs))
    actual = _flat(n["ModelNew"](*init)(*inputs))
    torch.cuda.synchronize()
    assert len(expected) == len(actual)
    for e, a in zip(expected, actual):
        assert e.shape == a.shape and e.dtype == a.dtype
        e32, a32 = e.float(), a.float()
        assert bool(torch.isfinite(a32).all())
        err = (e32 - a32).abs().max().item()
        ok = torch.allclose(e32, a32, atol=r["output_atol"], rtol=r["output_rtol"])
        assert ok, f"{name}: max abs error {err}"
