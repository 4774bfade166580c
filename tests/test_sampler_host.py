"""Host-side sampler functions of the C ABI against the oracle, bit-exact (no GPU needed):
LTX2Scheduler::execute (scheduler.rs:67-125) and the position grids
(patchifier.rs:101-161, 183-332)."""
import numpy as np
import pytest

from oracle import sampler


@pytest.mark.parametrize("steps,tokens", [(5, 1024), (8, 6144), (30, 6144), (40, 4096), (1, 1), (0, 10), (10, 100000)])
def test_scheduler_bit_exact(steps, tokens):
    import ltx_b200
    got = ltx_b200.scheduler_execute(steps, tokens)
    exp = sampler.scheduler_execute(steps, tokens)
    assert got.view(np.uint32).tolist() == exp.view(np.uint32).tolist()
    got = ltx_b200.scheduler_execute(steps, tokens, stretch=False)
    exp = sampler.scheduler_execute(steps, tokens, stretch=False)
    assert got.view(np.uint32).tolist() == exp.view(np.uint32).tolist()


def test_scheduler_known_values():
    import ltx_b200
    np.testing.assert_allclose(ltx_b200.scheduler_execute(5, 1024), [1.0, 0.8694, 0.6963, 0.4560, 0.1, 0.0], atol=1e-3)


@pytest.mark.parametrize("F,H,W,batch,fps", [(16, 24, 16, 1, 24.0), (3, 2, 2, 2, 24.0), (1, 1, 1, 1, 30.0),
                                              (5, 4, 3, 1, 12.5)])
def test_target_positions_bit_exact(F, H, W, batch, fps):
    import ltx_b200
    got = ltx_b200.target_positions(F, H, W, batch, fps=fps)
    exp = sampler.target_positions(F, H, W, batch, fps=fps)
    assert got.shape == exp.shape and (got.view(np.uint32) == exp.view(np.uint32)).all()


@pytest.mark.parametrize("F,H,W,first,tsf,ds", [(16, 24, 16, 0, 1, 1), (3, 2, 2, 1, 4, 2), (2, 3, 5, 7, 2, 3)])
def test_reference_positions_bit_exact(F, H, W, first, tsf, ds):
    import ltx_b200
    got = ltx_b200.reference_positions(F, H, W, 1, first, temporal_scale_factor=tsf, downscale_factor=ds)
    exp = sampler.reference_positions(F, H, W, 1, first, temporal_scale_factor=tsf, downscale_factor=ds)
    assert (got.view(np.uint32) == exp.view(np.uint32)).all()
