"""PLY export (trainer.py:570-631) byte for byte against the oracle's
restatement of the reference exporter, and checkpoint / resume of the whole
training state."""
import os

import numpy as np
import pytest
import torch

from mlx_gsplat_b200.trainer import runner_for_workload
from oracle import export as oexport

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("wl_name,n", [("tiny-3k", 3000), ("outdoor-1m", 5000)])
def test_export_to_ply_matches_reference_exporter(tmp_path, wl_name, n):
    r = runner_for_workload(wl_name, max_steps=10, n=n, num_views=4)
    al, L = r.allocator, r.layout
    # edge values: scales and opacities beyond the clip ranges, a NaN scale, a zero quaternion
    phys = al.indirection_table[:8].long()
    th = al.theta
    th[phys[0], L.offsets["scales"]] = 3.0
    th[phys[1], L.offsets["scales"] + 1] = -20.0
    th[phys[2], L.offsets["opacities"]] = 9.0
    th[phys[3], L.offsets["opacities"]] = -9.0
    th[phys[4], L.offsets["scales"] + 2] = float("nan")
    th[phys[5], L.quat_col:L.quat_col + 4] = 0.0
    r.train_step(0, 1)  # a trained state, not just the initial one
    path = os.path.join(tmp_path, "out.ply")
    count = r.export_to_ply(path)
    assert count == al.num_active
    theta = al.theta.cpu().numpy()[al.indirection_table.cpu().numpy()]
    active = {k: theta[:, o:o + L.dims[k]] for k, o in L.offsets.items()}
    ref = oexport.ply_bytes(active)
    got = open(path, "rb").read()
    assert len(got) == len(ref)
    assert got == ref


def test_checkpoint_resume_continues_the_run(tmp_path):
    a = runner_for_workload("tiny-3k", max_steps=20, n=3000, num_views=4, lr=1e-2)
    for step in range(1, 3):
        a.train_step(step - 1, step)
    path = os.path.join(tmp_path, "ckpt.npz")
    a.save_checkpoint(path)
    b = runner_for_workload("tiny-3k", max_steps=20, n=3000, num_views=4, lr=1e-2, seed=7)
    b.load_checkpoint(path)
    al, bl = a.allocator, b.allocator
    for k in ("theta", "adam_m", "adam_v", "indirection_table", "free_stack", "grad2d", "count"):
        assert torch.equal(getattr(al, k), getattr(bl, k)), k
    assert (al.free_top, a.optimizer.t, a.step_count) == (bl.free_top, b.optimizer.t, b.step_count)
    for r in (a, b):
        r.train_step(2, 3)
    torch.cuda.synchronize()
    # the rasterizer's gradient sums are float atomics: a few ulp between runs
    np.testing.assert_allclose(al.theta.cpu().numpy(), bl.theta.cpu().numpy(), rtol=1e-5, atol=1e-6)


def test_checkpoint_rejects_another_layout(tmp_path):
    a = runner_for_workload("tiny-3k", max_steps=5, n=3000, num_views=2)
    path = os.path.join(tmp_path, "ckpt.npz")
    a.save_checkpoint(path)
    b = runner_for_workload("outdoor-1m", max_steps=5, n=3000, num_views=2)
    with pytest.raises(ValueError):
        b.load_checkpoint(path)
