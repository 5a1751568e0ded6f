"""Self-tests of the test kit and of the distributed spawner (CPU, gloo).

Behaviour mirrors the reference's harness tests (tests/utils/test_testing.py):
clones, the mismatch budget, forward/backward comparison, spawner argument and
environment plumbing, failure propagation and teardown."""

import os
import socket
import time

import pytest
import torch
from torch.multiprocessing.spawn import ProcessRaisedException

from dtensor_muon_b200.testing.distributed import free_port
from testkit import as_tensors, assert_close, check_impls, clone_args, print_times, run_distributed


# ------------------------------------------------------------------ clones --
def test_clone_args_copies_tensors_keeps_requires_grad_and_shares_the_rest():
    t = torch.randn(3, 2, requires_grad=True)
    tag = object()
    a, b = clone_args((t, tag))
    assert a is not t and a.requires_grad and b is tag
    with torch.no_grad():
        a.mul_(0)
    assert t.abs().sum() > 0
    c, _ = clone_args((t, tag))
    assert c is not a


# ------------------------------------------------------------ assert_close --
def test_assert_close_compares_low_precision_in_fp32():
    x = torch.ones(16, dtype=torch.bfloat16)
    assert_close(x, torch.ones(16), rtol=0, atol=0)


def test_assert_close_strict_raises_on_one_bad_element():
    e = torch.zeros(100)
    a = e.clone()
    a[7] = 1.0
    with pytest.raises(AssertionError):
        assert_close(a, e, rtol=0, atol=1e-3)


def test_assert_close_budget_boundary_and_message():
    e = torch.zeros(100)
    a = e.clone()
    a[:2] = 1.0  # 2 % mismatched
    assert_close(a, e, rtol=0, atol=1e-3, max_mismatch_pct=2.0)
    with pytest.raises(AssertionError, match=r"(?s)ctx.*2\.0000% of elements mismatched"):
        assert_close(a, e, rtol=0, atol=1e-3, max_mismatch_pct=1.0, msg="ctx")


def test_assert_close_budget_on_empty_and_shape_mismatch():
    assert_close(torch.empty(0), torch.empty(0), max_mismatch_pct=0.0)
    with pytest.raises(AssertionError, match="shape"):
        assert_close(torch.zeros(2), torch.zeros(3), max_mismatch_pct=1.0)


def test_as_tensors_normalises_and_rejects():
    t = torch.zeros(1)
    assert as_tensors(t) == [t]
    assert as_tensors((t, t)) == [t, t]
    with pytest.raises(TypeError):
        as_tensors((t, 3))


# ------------------------------------------------------------ check_impls --
def _scale2(x):
    return x * 2


def test_check_impls_matching_passes_and_does_not_time_on_cpu():
    assert check_impls(_scale2, lambda x: x + x, (torch.randn(8),), bench=False) == {}


def test_check_impls_diverging_names_the_impl():
    with pytest.raises(AssertionError, match="wrong"):
        check_impls({"wrong": lambda x: x * 3}, _scale2, (torch.randn(8),), bench=False)


def test_check_impls_output_count_mismatch():
    with pytest.raises(AssertionError, match="outputs"):
        check_impls(lambda x: (x, x), _scale2, (torch.randn(4),), bench=False)


def test_check_impls_extra_baselines_are_checked_against_the_first():
    ok = {"ref": _scale2, "also": lambda x: 2 * x}
    check_impls({}, ok, (torch.randn(4),), bench=False)
    with pytest.raises(AssertionError, match="bad_base"):
        check_impls({}, {"ref": _scale2, "bad_base": lambda x: x}, (torch.randn(4),), bench=False)


def test_check_impls_every_impl_is_checked():
    impls = {"a": _scale2, "b": lambda x: x.mul(2), "c": lambda x: x + 1}
    with pytest.raises(AssertionError, match="c: output"):
        check_impls(impls, _scale2, (torch.randn(4),), bench=False)


def test_check_impls_gives_each_callable_its_own_inputs():
    x = torch.ones(4)

    def inplace(t):
        return t.add_(1)

    check_impls({"inplace": inplace}, lambda t: t + 1, (x,), bench=False)
    assert torch.equal(x, torch.ones(4))


def test_check_impls_backward_matches():
    x = torch.randn(5, requires_grad=True)
    check_impls(lambda t: t.square(), lambda t: t * t, (x,), bwd=True, bench=False)


def test_check_impls_backward_gradient_presence_mismatch():
    x, y = torch.randn(3, requires_grad=True), torch.randn(3, requires_grad=True)
    with pytest.raises(AssertionError, match="present"):
        check_impls(lambda a, b: a * 1 + b.detach(), lambda a, b: a + b, (x, y), bwd=True, bench=False)


def test_check_impls_backward_gradient_value_mismatch():
    x = torch.randn(6, requires_grad=True)
    # same forward values, different gradient (straight-through vs real)
    with pytest.raises(AssertionError, match="gradient of input 0"):
        check_impls(lambda t: t + (t * t - t * t.detach()), lambda t: t, (x,), bwd=True, bench=False)


def test_check_impls_backward_needs_a_grad_input():
    with pytest.raises(AssertionError, match="requires_grad"):
        check_impls(_scale2, _scale2, (torch.randn(3),), bwd=True, bench=False)


def test_print_times_marks_the_reference(capsys):
    import sys

    print_times({"ref": 2.0, "fast": 1.0}, "ref", file=sys.stdout)
    out = capsys.readouterr().out.splitlines()
    assert out[0].startswith("* ref") and "2.00x" in out[1]


# ---------------------------------------------------------------- spawner --
def _noop(rank, world):
    assert 0 <= rank < world


def _fails(rank, world):
    raise AssertionError(f"rank {rank} failed on purpose")


def _args_kwargs(rank, world, word, *, number):
    assert word == "passed" and number == 7


def _env(rank, world):
    assert os.environ["RANK"] == str(rank) and os.environ["LOCAL_RANK"] == str(rank)
    assert os.environ["WORLD_SIZE"] == str(world) and os.environ["MASTER_ADDR"] == "127.0.0.1"
    assert int(os.environ["MASTER_PORT"]) > 0


def _slow_rank0(rank, world):
    if rank == 0:
        time.sleep(0.2)


def test_free_port_is_bindable():
    port = free_port()
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", port))


@pytest.mark.parametrize("world", [1, 2, 3])
def test_spawner_runs_every_rank(world):
    run_distributed(_noop, world)


def test_spawner_propagates_a_worker_failure():
    with pytest.raises(ProcessRaisedException, match="failed on purpose"):
        run_distributed(_fails, 2)


def test_spawner_forwards_args_and_kwargs():
    run_distributed(_args_kwargs, 2, args=("passed",), kwargs={"number": 7})


def test_spawner_sets_the_rank_environment():
    run_distributed(_env, 2)


def test_spawner_is_reusable_after_a_failure():
    with pytest.raises(ProcessRaisedException):
        run_distributed(_fails, 2)
    run_distributed(_noop, 2)


def test_spawner_teardown_barrier_tolerates_uneven_ranks():
    run_distributed(_slow_rank0, 2)


@pytest.mark.gpu
def test_time_cuda_returns_positive_ms():
    from testkit import time_cuda

    x = torch.randn(1 << 20, device="cuda")
    assert time_cuda(lambda: x.mul_(1.0), reps=3) > 0.0
