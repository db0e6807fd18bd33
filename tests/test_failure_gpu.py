"""Failure detection without a GPU fault: every device-side wait of the
decode GEMM is bounded, and on timeout the kernel records AOS_ERR_TIMEOUT,
returns, and the host reads the status after the launch.  Here a kernel
runs the GEMM kernel's own wait routines (the grid barriers' counter spin
and the pipeline's mbarrier wait) against conditions nothing satisfies; each
must end by its time limit (about a second) with AOS_ERR_TIMEOUT, and the
context must stay usable: the next decode step equals a fresh context's."""
import time

import numpy as np
import pytest

from tests.aos_import import aos
from tests.test_decoder_gpu import Setup

pytestmark = pytest.mark.gpu

AOS_ERR_TIMEOUT = -6


def test_bounded_waits_time_out_and_the_context_stays_usable():
    s = Setup(seed=3)
    L = aos.lib()
    for kind in (0, 1):
        t0 = time.time()
        rc = L.aos_debug_bounded_wait(s.gpu.ctx, kind)
        dt = time.time() - t0
        assert rc == AOS_ERR_TIMEOUT, (kind, rc)
        assert "timed out" in aos.last_error(s.gpu.ctx)
        assert 0.2 < dt < 20.0, dt
    s.gpu.health_check()
    logits, hidden = s.gpu.run_step_batch(s.rings, s.tokens.astype(np.uint32), s.seq_ids, want_hidden=True)
    fresh = Setup(seed=3)
    ref_logits, ref_hidden = fresh.gpu.run_step_batch(fresh.rings, fresh.tokens.astype(np.uint32), fresh.seq_ids,
                                                      want_hidden=True)
    assert logits.tobytes() == ref_logits.tobytes() and hidden.tobytes() == ref_hidden.tobytes()
    s.gpu.close()
    fresh.gpu.close()
