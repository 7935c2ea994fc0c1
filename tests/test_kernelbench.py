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


def _set_seed(seed):
    torch.manual_seed(seed)
    torch.cuda.manual_seed(seed)


def _kernelevo_trial(name, precision, seed=42, trial_seed=1234):
    """One correctness trial the way KernelEvo runs it (eval.py:418-439, 590-606, 840-900):
    seeded construction of both models, ``.to(device, dtype=precision)``, seeded inputs cast
    to ``precision`` on the device, ``torch.allclose`` on the single output."""
    ref, new = kernelbench.task_source(name)
    r, n = _load(ref), _load(new)
    dev = torch.device("cuda", 0)
    init = r["get_init_inputs"]()
    _set_seed(seed)
    model = r["Model"](*init)
    _set_seed(seed)
    model_new = n["ModelNew"](*init)
    model = model.to(device=dev, dtype=precision)
    model_new = model_new.to(device=dev, dtype=precision)
    _set_seed(trial_seed)
    inputs = [x.to(dtype=precision).to(device=dev) if torch.is_tensor(x) else x
              for x in r["get_inputs"]()]
    with torch.no_grad():
        expected = model(*inputs)
        actual = model_new(*inputs)
    torch.cuda.synchronize()
    assert expected.shape == actual.shape
    e32, a32 = expected.float(), actual.float()
    assert bool(torch.isfinite(a32).all())
    err = (e32 - a32).abs().max().item()
    ok = torch.allclose(e32, a32, atol=r["output_atol"], rtol=r["output_rtol"])
    return ok, err


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(kernelbench.TASKS))
def test_model_new_matches_model(name):
    ok, err = _kernelevo_trial(name, torch.float32)
    assert ok, f"{name}: max abs error {err}"


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["gemm_bias_relu_fp8", "gpt2_block_fp8"])
def test_model_new_matches_model_bf16_precision(name):
    ok, err = _kernelevo_trial(name, torch.bfloat16)
    assert ok, f"{name}: max abs error {err}"
