"""Command line of the trainer, with the reference's flags and defaults
(train.py:11-23): ``python -m mlx_gsplat_b200.train --data_dir data/garden``.

Builds an ``MLXConfig`` from the flags, trains (a COLMAP scene under
``--data_dir``, or the reference's synthetic mode when there is none) and
writes ``<scene>_mlx_custom_3dgs.ply`` at the end, as the reference does.
Flags the reference does not have: ``--loss``, ``--sh_eval``, ``--seed``,
``--no_export``.
"""
from __future__ import annotations

import argparse
from typing import List, Optional

from .trainer import MLXConfig, RunnerMLX


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="B200 3DGS trainer")
    ap.add_argument("--data_dir", type=str, default="data/garden", help="COLMAP scene directory")
    ap.add_argument("--max_steps", type=int, default=2500, help="training steps")
    ap.add_argument("--sh_degree_interval", type=int, default=500, help="steps per SH degree of the schedule")
    ap.add_argument("--data_factor", type=int, default=4, help="image downscale factor")
    ap.add_argument("--render_width", type=int, default=200, help="render width")
    ap.add_argument("--render_height", type=int, default=150, help="render height")
    ap.add_argument("--pixel_chunk_size", type=int, default=1024,
                    help="accepted for compatibility (the tile rasterizer does not chunk pixels)")
    ap.add_argument("--max_gaussians", type=int, default=500000, help="fixed pool capacity")
    ap.add_argument("--init_gaussians", type=int, default=None, help="cap on the initial SfM points")
    ap.add_argument("--lazy_images", action="store_true", help="decode each step's image instead of preloading")
    ap.add_argument("--loss", choices=["l1+dssim", "l1", "mean"], default="l1+dssim",
                    help="image loss (the reference trainer's 0.8 L1 + 0.2 D-SSIM by default)")
    ap.add_argument("--sh_eval", choices=["reference", "full"], default="reference",
                    help="SH colour: the reference's degree <= 1, or real SH up to degree 3")
    ap.add_argument("--seed", type=int, default=0, help="seed of the random draws")
    ap.add_argument("--no_export", action="store_true", help="do not write the PLY at the end")
    return ap


def config_from_args(args: argparse.Namespace) -> MLXConfig:
    cfg = MLXConfig()
    cfg.data_dir = args.data_dir
    cfg.max_gaussians = args.max_gaussians
    cfg.init_gaussians = args.init_gaussians
    cfg.max_steps = args.max_steps
    cfg.sh_degree_interval = args.sh_degree_interval
    cfg.data_factor = args.data_factor
    cfg.render_width = args.render_width
    cfg.render_height = args.render_height
    cfg.pixel_chunk_size = args.pixel_chunk_size
    cfg.preload_images = not args.lazy_images
    cfg.loss = args.loss
    cfg.sh_eval = args.sh_eval
    cfg.seed = args.seed
    cfg.export_ply_on_finish = not args.no_export
    return cfg


def main(argv: Optional[List[str]] = None) -> RunnerMLX:
    cfg = config_from_args(build_parser().parse_args(argv))
    runner = RunnerMLX(cfg)
    runner.train()
    return runner


if __name__ == "__main__":
    main()
