"""The trainer's command line (the reference's train.py flags and defaults),
checked on the CPU: flags map onto the config fields the trainer reads."""
from mlx_gsplat_b200 import train
from mlx_gsplat_b200.trainer import MLXConfig


def test_defaults_follow_the_reference_cli():
    cfg = train.config_from_args(train.build_parser().parse_args([]))
    assert (cfg.data_dir, cfg.max_steps, cfg.sh_degree_interval, cfg.data_factor) == ("data/garden", 2500, 500, 4)
    assert (cfg.render_width, cfg.render_height, cfg.max_gaussians, cfg.init_gaussians) == (200, 150, 500000, None)
    assert cfg.preload_images and cfg.export_ply_on_finish
    assert cfg.loss == "l1+dssim" and cfg.sh_eval == "reference"


def test_flags_reach_the_config():
    args = train.build_parser().parse_args(
        ["--data_dir", "scene", "--max_steps", "7", "--sh_degree_interval", "3", "--data_factor", "2",
         "--render_width", "64", "--render_height", "48", "--max_gaussians", "1000", "--init_gaussians", "10",
         "--lazy_images", "--loss", "l1", "--sh_eval", "full", "--seed", "5", "--no_export"])
    cfg = train.config_from_args(args)
    assert isinstance(cfg, MLXConfig)
    assert (cfg.data_dir, cfg.max_steps, cfg.sh_degree_interval, cfg.data_factor) == ("scene", 7, 3, 2)
    assert (cfg.render_width, cfg.render_height, cfg.max_gaussians, cfg.init_gaussians) == (64, 48, 1000, 10)
    assert not cfg.preload_images and not cfg.export_ply_on_finish
    assert (cfg.loss, cfg.sh_eval, cfg.seed) == ("l1", "full", 5)
