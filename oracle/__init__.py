"""CPU checkers for the parity tests (test infrastructure, never the product path).

* ``oracle.display`` -- ctypes wrapper of ``liboracle.so``, the C restatement of the
  reference's display-path stages (project, tile_assign, sort_and_bin, blend), and a
  loader for ``oracle/_ref``, the reference's own CPU pipeline compiled from its sources.
* ``oracle.train`` -- numpy restatement of the reference's training-path models
  (tiled fp32 forward, L1/SSIM loss, blend backward, projection backward incl. SH1-3,
  sparse Adam).
* ``oracle.train_pool`` -- the oracle's multi-view training step with one view per
  spawned worker process (the CPU baseline on all host cores).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use
this package.
"""
