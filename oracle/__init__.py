"""CPU oracle for the 3DGS training hot path — TEST INFRASTRUCTURE ONLY.

A plain restatement, on the CPU, of the reference's algorithm for each piece
of the hot path, used only as the checker by ``tests/``, by
``__graft_entry__.smoke()`` and by the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``.  The product (``mlx_gsplat_b200``) never imports it and
has no CPU fallback.

Modules and the reference code each one follows:

* ``oracle.rendering`` — ``frustum_culling_mlx`` (``mlx_gsplat/rendering.py:41-94``)
  and the dense differentiable rasterizer ``rasterize_gaussians_mlx``
  (``mlx_gsplat/rendering.py:97-308``), with MLX's autograd restated through
  torch-CPU autograd plus MLX's clip/maximum gradient tie rules.
* ``oracle.adam`` — the fused Metal Adam (``src/mlx_extensions.cpp:102-152``,
  restated in C in ``oracle/adam_a1.c``) and the pure-MLX Adam
  (``mlx_gsplat/optimizer.py:146-175``).
* ``oracle.allocator`` — ``PointerStableChunkedAllocator``
  (``mlx_gsplat/allocator.py:8-292``), including its LIFO free-list order.
* ``oracle.densify`` — the trainer's densify/prune policy and child values
  (``mlx_gsplat/trainer.py:421-519``), the grad2d proxy (``:300-318``), the
  quaternion renorm (``:380-387``) and the opacity reset (``:416-419``).

Pinning: the reference's own Python files are executed over a torch-CPU
stand-in for ``mlx.core`` by ``tests/golden/gen_golden.py``; the fixtures it
writes under ``tests/golden/`` pin these restatements
(``tests/test_oracle_golden.py``).  The Metal Adam source is compiled as C++
from the reference file itself by ``oracle/build_ref.py`` into ``oracle/_ref``
and pins ``adam_a1.c``.
"""
