"""CPU check of the stencil forward's mbarrier protocol (model in tests/stencil_protocol.py).

The kernel's producer / MMA / softmax roles are replayed under many random
interleavings with the hardware's parity-wait semantics.  The shipped barrier map must
survive all of them; the earlier stage-release scheme, which let the producer pass its
first release waits before the MMAs had finished with the stage, and the broken variants
of the two-P-buffer scheme must be caught.
"""
import pytest

import stencil_protocol as sp


@pytest.mark.parametrize("stages", [3, 4])
@pytest.mark.parametrize("n_chunks", [10, 15])
def test_forward_protocol_holds_under_random_interleavings(stages, n_chunks):
    for seed in range(150):
        sp.run_fwd(n_chunks=n_chunks, stages=stages, seed=seed)


def test_model_rejects_overwriting_s_before_the_warps_load_it():
    failures = 0
    for seed in range(100):
        try:
            sp.run_fwd(n_chunks=12, stages=4, seed=seed, skip_sfree=True)
        except sp.ProtocolError as err:
            assert "before the softmax warps loaded it" in str(err) or "overwritten before" in str(err)
            failures += 1
    assert failures > 0


def test_model_rejects_one_p_buffer_without_a_wait():
    """With a single P buffer, storing P(c) needs PV(c - 1) to have completed; the kSFull
    commit that covers the two-buffer scheme does not cover that."""
    failures = 0
    for seed in range(100):
        try:
            sp.run_fwd(n_chunks=12, stages=4, seed=seed, p_buffers=1)
        except sp.ProtocolError as err:
            assert "may read it" in str(err)
            failures += 1
    assert failures > 0


def test_model_rejects_kpfree_waits_on_rescale_only():
    """Skipping the wait for PV(c - 1) on every chunk without a rescale lets kPFree run more
    than one completion ahead of a later parity wait."""
    failures = 0
    for seed in range(300):
        try:
            sp.run_fwd(n_chunks=12, stages=4, seed=seed, wait_on_rescale_only=True)
        except sp.ProtocolError as err:
            assert "passed at" in str(err) or "before PV" in str(err)
            failures += 1
    assert failures > 0


def test_two_tile_protocol_with_release_barriers_holds():
    """The earlier two-tile forward, repaired with per-stage release barriers."""
    for seed in range(100):
        sp.run(n_chunks=14, stages=4, seed=seed, release="empty")


def test_model_rejects_the_ambiguous_release_scheme():
    failures = 0
    for seed in range(100):
        try:
            sp.run(n_chunks=14, stages=4, seed=seed, release="sready")
        except sp.ProtocolError as err:
            assert "passed at 0" in str(err)
            failures += 1
    assert failures > 0


@pytest.mark.parametrize("stages", [2, 3, 4])
def test_dq_protocol_holds_under_random_interleavings(stages):
    for seed in range(150):
        sp.run_dq(n_chunks=12, stages=stages, seed=seed)


@pytest.mark.parametrize("sep_p", [True, False])
@pytest.mark.parametrize("stages", [2, 4, 8])
@pytest.mark.parametrize("n_chunks", [1, 2, 3, 14])
def test_dkv_protocol_holds(sep_p, stages, n_chunks):
    """dK / dV kernels at two CTAs per SM: dS^T over dP^T, P^T over S^T or in a buffer of its
    own, tensor-core operations ordered only per accumulator."""
    for seed in range(80):
        sp.run_ip(n_chunks=n_chunks, stages=stages, seed=seed, sep_p=sep_p)


def test_model_rejects_issuing_the_next_scores_before_the_products_complete():
    failures = 0
    for seed in range(150):
        try:
            sp.run_ip(n_chunks=10, stages=4, seed=seed, sep_p=seed % 2 == 0, skip_accdone=True)
        except sp.ProtocolError as err:
            assert "before dV/dK" in str(err) or "read lanes" in str(err) or "lanes hold" in str(err)
            failures += 1
    assert failures > 0
