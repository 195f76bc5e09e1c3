"""The GPU ImportanceMigrator against the reference's ImportanceBasedMigrator
(akv/vmm.py:113-245), replayed from a trace recorded by running the
reference (tests/golden/make_golden.py: make_migrator_trace): seeded
attention per step over a growing sequence, promotion marks, and the
importance vector and eviction candidates at several steps."""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def test_migrator_trace_matches_reference(golden_dir):
    from akv.tiering import ImportanceMigrator
    z = np.load(os.path.join(golden_dir, "migrator.npz"))
    mig = ImportanceMigrator(importance_decay=0.9, protect_initial=4, protect_recent=32, device=DEV)
    checked = 0
    for step in range(40):
        attn = torch.from_numpy(z[f"attn{step}"]).to(DEV)
        N = attn.shape[-1]
        mig.update(0, attn, N)
        if f"promote{step}" in z:
            mig.mark_promoted(0, torch.from_numpy(z[f"promote{step}"]).to(DEV))
        if f"imp{step}" in z:
            imp = mig.compute_importance(0, N).cpu().numpy()
            np.testing.assert_array_equal(imp.view(np.uint32), z[f"imp{step}"].view(np.uint32), err_msg=f"step {step}")
            ev = mig.get_eviction_candidates(0, N, 50).cpu().numpy()
            np.testing.assert_array_equal(ev, z[f"evict{step}"], err_msg=f"step {step}")
            checked += 1
        mig.advance_step()
    assert checked == 8


def test_migrator_protects_everything_when_short():
    from akv.tiering import ImportanceMigrator
    mig = ImportanceMigrator(protect_initial=4, protect_recent=32, device=DEV)
    a = torch.softmax(torch.randn(1, 2, 1, 30, device=DEV), -1)
    mig.update(0, a, 30)
    assert torch.isinf(mig.compute_importance(0, 30)).all()
    assert mig.get_eviction_candidates(0, 30, 10).numel() == 0
    mig.reset()
    assert torch.equal(mig.compute_importance(0, 5).cpu(), torch.arange(5, dtype=torch.float32))
