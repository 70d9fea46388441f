"""Failure detection without a GPU fault: a bounded wait in the persistent
decode kernel is made to run out (a grid-barrier arrival that nothing
provides); the host must get SLM_ERR_DEVICE and the context must stay usable."""
import time

import numpy as np
import pytest

from conftest import load_pkg

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def small_model(tmp_path_factory):
    load_pkg()
    syn = __import__("slm_b200.synthetic").synthetic
    cfg = syn.scaled(syn.BASE, vocab_size=500, d_model=128, n_heads=2, hidden=256, window=32, max_loops=2,
                     default_loops=2)
    return syn.write_model(tmp_path_factory.mktemp("stall"), cfg, seed=9)


def test_expired_wait_is_reported_and_the_context_survives(slm, ctx, small_model):
    model = slm.Model(ctx, small_model)
    ids = np.arange(40) % 500
    ref = model.session()
    ref.feed(ids)
    ref.step(7)
    want = ref.logits()

    bad = model.session()
    assert bad.mega
    bad.feed(ids)
    bad.set_stall_test(True)
    t0 = time.time()
    bad.step(7)  # queued; the kernel gives up after its bounded wait
    with pytest.raises(slm.SlmError) as e:
        bad.logits()
    assert e.value.code == 5 and "bounded wait" in str(e.value)
    assert time.time() - t0 < 30

    # The context is still usable: a new session reproduces the good logits.
    good = model.session()
    good.feed(ids)
    good.step(7)
    np.testing.assert_allclose(good.logits(), want, atol=1e-6)


def test_expired_wait_reaches_the_sampler_not_a_stale_id(slm, ctx, small_model):
    # A greedy slm_sample right after slm_step polls the step's mailbox; a step
    # that gave up writes none, so the sampler must report the error once the
    # stream is idle (never the arg-max of an earlier step).
    model = slm.Model(ctx, small_model)
    ids = np.arange(40) % 500
    greedy = slm.Sampling()
    ref = model.session()
    ref.feed(ids)
    ref.step(7)
    want = ref.sample(greedy)

    bad = model.session()
    bad.feed(ids)
    bad.step(3)
    bad.sample(greedy)  # a good step first: its mailbox holds an id
    bad.set_stall_test(True)
    bad.step(7)
    with pytest.raises(slm.SlmError) as e:
        bad.sample(greedy)
    assert e.value.code == 5 and "bounded wait" in str(e.value)

    good = model.session()
    good.feed(ids)
    good.step(7)
    assert good.sample(greedy) == want
