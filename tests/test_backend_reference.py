"""B200Backend against the reference's own plugin interface, on the CPU (no GPU needed):
it subclasses the reference's Backend ABC (gsplat/backend.py:41-158) with the same stage
signatures, and the reference's Pipeline (gsplat/pipeline.py:131-260) drives it through
both of its paths -- the fused one (has_render_fused / render_fused) and the staged one
(project -> tile_assign -> sort -> blend) -- with every call binding to B200Backend's
signatures and every render knob the Pipeline pushes landing on an attribute the backend
has. The check runs in a child process with the reference project on sys.path; it is
skipped where the reference is absent (the reference root is $GSPLAT_TT_REFERENCE, else the
`reference_path` recorded in BASELINE.json)."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
from __graft_entry__ import reference_root  # noqa: E402

CHILD = r'''
import inspect, sys
import numpy as np
import torch
from gsplat.backend import Backend as RefBackend
from gsplat.data_structures import Gaussians
from gsplat.pipeline import Pipeline
from gsplat_tt_b200.backend import B200Backend

assert issubclass(B200Backend, RefBackend), "B200Backend does not subclass the reference ABC"
for name in ("project", "tile_assign", "sort", "blend", "close"):
    ref = inspect.signature(getattr(RefBackend, name))
    got = inspect.signature(getattr(B200Backend, name))
    rp = [(p.name, p.kind, p.default) for p in ref.parameters.values()]
    gp = [(p.name, p.kind, p.default) for p in got.parameters.values()]
    assert rp == gp, (name, rp, gp)

calls = []

class Recorder(B200Backend):
    """B200Backend's signatures and attributes; the stage bodies are the reference ABC's CPU
    defaults (no GPU here), so the Pipeline runs end to end."""
    def __init__(self, fused):
        self.tile_size = 16
        self._render_fused = fused
        self.cull_disabled = False
        self.min_opacity = self.max_radius = self.k_cap = None
        self.contrib_floor_override = self._mb_contrib_floor = None
        self.transmittance_threshold = None
        self.use_isoellipse = None
        self._cov3d = self._cov3d_key = None

    def _bind(self, name, args, kwargs):
        inspect.signature(getattr(B200Backend, name)).bind(self, *args, **kwargs)
        calls.append(name)

    def project(self, *a, **k):
        self._bind("project", a, k)
        return RefBackend.project(self, *a, **k)

    def tile_assign(self, *a, **k):
        self._bind("tile_assign", a, k)
        return RefBackend.tile_assign(self, *a, **k)

    def sort(self, *a, **k):
        self._bind("sort", a, k)
        return RefBackend.sort(self, *a, **k)

    def blend(self, *a, **k):
        self._bind("blend", a, k)
        H, W = a[6], a[7]
        return np.zeros((H, W, 3), np.float32), {}

    def render_fused(self, *a, **k):
        self._bind("render_fused", a, k)
        H, W = a[3], a[4]
        return np.zeros((H, W, 3), np.float32), {"num_visible": 1, "num_entries": 1}

rng = np.random.default_rng(0)
n = 300
q = rng.standard_normal((n, 4)).astype(np.float32)
q /= np.linalg.norm(q, axis=1, keepdims=True)
g = Gaussians(means=torch.from_numpy(rng.uniform(-1, 1, (n, 3)).astype(np.float32)),
              scales=torch.from_numpy(np.exp(rng.normal(-4, 0.5, (n, 3))).astype(np.float32)),
              rotations=torch.from_numpy(q),
              colors=torch.from_numpy(rng.uniform(0, 1, (n, 3)).astype(np.float32)),
              opacities=torch.from_numpy(rng.uniform(0.2, 1, n).astype(np.float32)))
E = torch.eye(4); E[2, 3] = 3.0
K = torch.tensor([[80.0, 0, 32], [0, 80.0, 32], [0, 0, 1]])
for fused in (True, False):
    b = Recorder(fused)
    p = Pipeline(b, tile_size=16, min_opacity=0.01, max_radius=5, k_cap=2.5)
    assert (b.min_opacity, b.max_radius, b.k_cap) == (0.01, 5, 2.5), "render knobs not pushed"
    calls.clear()
    res = p.render(g, E, K, 64, 64)
    assert res.image.shape == (64, 64, 3)
    want = ["render_fused"] if fused else ["project", "tile_assign", "sort", "blend"]
    assert calls == want, (fused, calls)
print("ok")
'''


@pytest.mark.skipif(reference_root() is None, reason="the reference project is not present")
def test_b200_backend_is_a_reference_backend_and_drives_the_reference_pipeline():
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([reference_root(), ROOT, env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", CHILD], capture_output=True, text=True, env=env,
                       cwd=ROOT, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
