"""The bounded waits on a B200: a wait that runs out is reported, never silent, and leaves the
context usable.  The wait that runs out is the test entry point's (lrs_test_wait_timeout: an
mbarrier phase that nothing completes, the wait primitive of every wait in the sampling
kernel, a bound of 20,000 cycles); no copy is in flight and no other thread waits on it."""
import numpy as np
import pytest

import lrs
from lrs import workloads as W
from gpu_util import run_oracle


@pytest.mark.gpu
def test_bounded_wait_runs_out_and_the_context_stays_usable():
    import torch
    w = W.headline(row_ids=range(0, 1024, 128))
    bs = lrs.BatchSampler(len(w.params), w.vocab, w.window)
    bs.set_params(w.params)
    bs.set_state(w.state)
    rtok, rinfo, rst = run_oracle(w.logits, w.vocab, w.hist, w.hist_len, w.params, w.state)
    # reported by lrs_poll_error, then cleared
    bs.test_wait_timeout(20_000)
    with pytest.raises(lrs.SamplerError) as ei:
        bs.poll_error()
    assert ei.value.code == lrs.LRS_E_TIMEOUT
    bs.poll_error()
    tok, probs = bs.sample(w.logits, hist=w.hist, hist_len=w.hist_len, probs=True)
    np.testing.assert_array_equal(tok, rtok)
    np.testing.assert_array_equal(bs.get_state(len(w.params)), rst)
    # reported by the next call on the context once it is known on the host (that call is
    # not enqueued: the state stays where it was)
    bs.set_state(w.state)
    bs.test_wait_timeout(20_000)
    torch.cuda.synchronize()
    with pytest.raises(lrs.SamplerError) as ei:
        bs.sample(w.logits, hist=w.hist, hist_len=w.hist_len)
    assert ei.value.code == lrs.LRS_E_TIMEOUT
    np.testing.assert_array_equal(bs.get_state(len(w.params)), w.state)
    tok = bs.sample(w.logits, hist=w.hist, hist_len=w.hist_len)
    tok = tok[0] if isinstance(tok, tuple) else tok
    np.testing.assert_array_equal(tok, rtok)
    bs.poll_error()
    bs.close()
