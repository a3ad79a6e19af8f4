"""Kernel-side failures reach the host as DtaError, on a GPU, without any
faulting or hanging input: a test hook makes every CTA's producer wait on a
barrier that nothing completes, so that bounded wait runs out after a short
budget and the kernel returns through its abort path; out-of-range explicit
rows are clamped and flagged.  The context must stay usable afterwards."""

import pytest
import torch

from delta_attention_b200.synthetic import make_inputs
from oracle import delta_oracle as orc
from tests._helpers import assert_close

pytestmark = pytest.mark.gpu

SHORT_WAIT = 2_000_000  # clock64 cycles, about a millisecond


def _inputs():
    q, k, v = make_inputs(1024, 8, 2, 128, seed=2)
    return q.cuda(), k.cuda(), v.cuda(), (q, k, v)


def test_stalled_wait_runs_out_and_is_reported():
    from delta_attention_b200 import ops
    from delta_attention_b200._lib import FLAG_TEST_STALL, DtaError
    q, k, v, cpu = _inputs()
    ops.check_errors()  # start clean
    ops.prefill(q, k, v, gamma=64, window=256, sink=64, flags=FLAG_TEST_STALL, wait_cycles=SHORT_WAIT)
    with pytest.raises(DtaError, match=r"KERNEL_TIMEOUT.*code 10[123]"):
        ops.check_errors()
    # the word was cleared, the context works: a normal call is correct
    out = ops.prefill(q, k, v, gamma=64, window=256, sink=64, check=True)
    ref = orc.delta_forward(*(t.float() for t in cpu), 64, 256, 64)
    assert_close(out.cpu(), ref, "prefill after a timed-out launch")


def test_stalled_wait_in_workspace_header():
    """Without the caller's error word the code lands in the workspace header,
    which dta_check_workspace reads."""
    from delta_attention_b200 import ops
    from delta_attention_b200._lib import FLAG_TEST_STALL, DtaError
    q, k, v, _ = _inputs()
    ws = ops.prefill_workspace(1, 8, 2, 1024, 128, gamma=64, window=256, sink=64, device=q.device)
    ops.prefill(q, k, v, gamma=64, window=256, sink=64, workspace=ws, use_error_word=False,
                flags=FLAG_TEST_STALL, wait_cycles=SHORT_WAIT, phases=1)
    with pytest.raises(DtaError, match="KERNEL_TIMEOUT"):
        ops.check_workspace(ws)
    ops.prefill(q, k, v, gamma=64, window=256, sink=64, workspace=ws, use_error_word=False, phases=1)
    assert ops.check_workspace(ws) == 0


def test_rows_stall_and_bad_rows_are_reported():
    from delta_attention_b200 import ops
    from delta_attention_b200._lib import FLAG_TEST_STALL, DtaError
    q, k, v, cpu = _inputs()
    rows = torch.tensor([0, 100, 1023])
    ops.rows(q, k, v, rows, rows, flags=FLAG_TEST_STALL, wait_cycles=SHORT_WAIT)
    with pytest.raises(DtaError, match="KERNEL_TIMEOUT"):
        ops.check_errors()
    # a query row past the end, bypassing the host check: clamped in the kernel and flagged
    ops.rows(q, k, v, torch.tensor([0, 1030]), torch.tensor([0, 10]), validate=False)
    with pytest.raises(DtaError, match="code 105"):
        ops.check_errors()
    with pytest.raises(ValueError):
        ops.rows(q, k, v, torch.tensor([0, 1030]), torch.tensor([0, 10]))
    out = ops.rows(q, k, v, rows, rows, check=True)
    ref = orc.dense_rows(cpu[0].float(), cpu[1].float(), cpu[2].float(), rows, 128 ** -0.5)
    assert_close(out.cpu(), ref, "rows after flagged calls")
