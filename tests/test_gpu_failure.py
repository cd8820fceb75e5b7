"""Failure detection on the GPU without a fault.

Every kernel of the library bounds its waits: a wait that runs out sets the
device-side error word's timeout bit, the kernel returns, and the host turns
the word into an error on its next check. Here a self-test kernel waits on a
barrier that nothing completes (the way a lost peer or a stalled producer
would leave a wait), with a limit of about a millisecond; the test checks
that the wait gave up, that the word says so and is cleared by the read, and
that the device still computes ref's bits afterwards.
"""
import pytest

from tests.cases import gemm_oracle, random_gemm_case


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_reports(pkb, cuda_device):
    pkb.device_errors(0)  # start from a clear word
    assert pkb.wait_selftest(2_000_000) is True
    assert pkb.device_errors(0) & 1  # PKB_DEVERR_TIMEOUT
    assert pkb.device_errors(0) == 0  # the read cleared it


@pytest.mark.gpu
def test_device_usable_after_a_wait_gave_up(pkb, oracle, cuda_device):
    assert pkb.wait_selftest(1_000_000) is True
    pkb.device_errors(0)
    case = random_gemm_case(7, 64, 256, 40, 32, add=True, bias=True, sliced=False)
    out = case["out"].copy()
    pkb.gemm_q8_host(out, case["os"], case["w_full"], case["ws_full"], case["bias_full"], case["rows_full"],
                     case["q"], case["d"], case["n"], case["qb"], case["T"], case["add"])
    assert (out.view("u4") == gemm_oracle(case).view("u4")).all()
    assert pkb.device_errors(0) == 0


def test_wait_selftest_refuses_bad_limits(pkb):
    with pytest.raises(pkb.PkbError):
        pkb.wait_selftest(10)
