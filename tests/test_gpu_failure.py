"""Device-side failure detection without a GPU fault: a bounded wait that runs
out.  qwen_debug_inject_wait shortens every wait on another CTA's values to
5 ms and makes the CTAs of one KV head withhold their layer-0 q|k|v, so their
peers' waits expire: the kernel records the error, stops waiting, drains its
copies and returns; the call reports QWEN_E_TIMEOUT, the device state is reset
and the KV cache invalidated.  The handle must then work again, at oracle
parity (max-abs <= 2e-2, relative RMS <= 2.5e-3)."""
import numpy as np
import pytest

from conftest import rel_rms

pytestmark = pytest.mark.gpu

VOCAB = 151936
PROMPT = np.random.default_rng(21).integers(0, VOCAB, 12).tolist()


@pytest.mark.parametrize("group", [0, 5])
def test_expired_wait_reports_timeout_and_handle_recovers(qb, O, checkpoint, group):
    eng = qb.Engine(checkpoint, 0)
    try:
        eng.prefill(PROMPT[:8], 0)
        eng.debug_inject_wait(5_000_000, group)
        with pytest.raises(qb.QwenError) as e:
            eng.decode_step(PROMPT[8], 8)
        assert e.value.code == -5, str(e.value)
        assert eng.cached == 0
        with pytest.raises(qb.QwenError) as e:      # the cache is gone: position 8 is no longer contiguous
            eng.decode_step(PROMPT[8], 8)
        assert e.value.code == -7
        eng.debug_inject_wait(0, -1)
        o = O.Oracle(checkpoint, O.FP32, 16)
        try:
            for pos, t in enumerate(PROMPT):
                lg = eng.forward(t, pos)
                lo = o.forward(t, pos)
                assert np.abs(lg - lo).max() <= 2e-2 and rel_rms(lg, lo) <= 2.5e-3, pos
        finally:
            o.close()
        nxt, _ = eng.decode_step(int(np.argmax(lg)), len(PROMPT))
        assert 0 <= nxt < VOCAB
    finally:
        eng.close()


def test_inject_wait_rejects_bad_arguments(qb, checkpoint, engine):
    with pytest.raises(qb.QwenError) as e:
        engine.debug_inject_wait(1000, -1)           # below 1 ms
    assert e.value.code == -1
    with pytest.raises(qb.QwenError) as e:
        engine.debug_inject_wait(0, 8)               # no such KV head
    assert e.value.code == -1
