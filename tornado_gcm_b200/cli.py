"""Command-line interface — reference ``cli.py:17-152`` (``train`` / ``infer`` / ``benchmark``).

The reference's commands call APIs it does not define (``SDAInference.from_state_dict``,
``.rollout``, ``load_initial_condition``, ``save_forecast``, ``PrecisionBenchmark``,
``trainer.train``); here they all exist.  Models are built from the config's
``model`` section (resolution), or converted from a NeuralGCM JAX checkpoint
with ``--jax-weights``.

    tornado-gcm-b200 train -c configs/sda_b200_2.8deg.yaml -k ckpt.pt -s 1000
    tornado-gcm-b200 infer -c configs/sda_b200_2.8deg.yaml -k ckpt.pt -i ic.pt -o forecast.npz -s 40
    tornado-gcm-b200 benchmark -c configs/sda_b200_2.8deg.yaml -s 2 -r report.txt
"""

from __future__ import annotations

import logging
import pathlib
from typing import Optional

import click

logger = logging.getLogger("tornado_gcm_b200")


def _config_path(path: str) -> str:
    p = pathlib.Path(path)
    if p.exists():
        return str(p)
    packaged = pathlib.Path(__file__).parent / "configs" / p.name
    if packaged.exists():
        return str(packaged)
    raise click.BadParameter(f"config {path} not found")


def _device(name: str) -> str:
    import torch

    if name.startswith("cuda") and not torch.cuda.is_available():
        logger.warning("CUDA not available; using the CPU")
        return "cpu"
    return name


@click.group()
@click.version_option(package_name="tornado_gcm_b200")
@click.option("--verbose", "-v", is_flag=True, help="Debug logging.")
def main(verbose: bool = False) -> None:
    """B200-native hybrid GCM with precision-zoned (PZHA) mixed precision."""
    logging.basicConfig(level=logging.DEBUG if verbose else logging.INFO,
                        format="%(asctime)s %(name)s %(levelname)s %(message)s")


@main.command()
@click.option("--config", "-c", required=True, help="SDA YAML config (path or packaged name).")
@click.option("--checkpoint", "-k", default=None, type=click.Path(), help="Checkpoint to resume from / save to.")
@click.option("--jax-weights", default=None, type=click.Path(exists=True),
              help="NeuralGCM JAX checkpoint to convert and initialise from.")
@click.option("--steps", "-s", default=None, type=int, help="Training steps (default: config).")
@click.option("--batch-size", "-b", default=None, type=int, help="Per-device batch (default: config).")
@click.option("--device", "-d", default="cuda", show_default=True)
@click.option("--use-sda/--no-sda", default=True, show_default=True, help="Drive phases with the SDA scheduler.")
@click.option("--parallel", type=click.Choice(["dp", "sharded"]), default="dp", show_default=True,
              help="Under torchrun: dp = replicated weights and optimizer, gradients averaged; sharded = "
                   "gradients and AdamW state split over the ranks.")
def train(config: str, checkpoint: Optional[str], jax_weights: Optional[str], steps: Optional[int],
          batch_size: Optional[int], device: str, use_sda: bool, parallel: str) -> None:
    """Train the hybrid model (synthetic reanalysis-shaped data unless the config names a source).

    Launched by torchrun with several processes, every rank trains on its own batches and the
    gradients are combined as ``--parallel`` says; rank 0 reports and writes the checkpoint."""
    from tornado_gcm_b200.models.builders import build_hybrid_gcm
    from tornado_gcm_b200.parallel.ddp import get_rank, setup_distributed
    from tornado_gcm_b200.precision.sda import SDAConfig
    from tornado_gcm_b200.training.sda_trainer import SDATrainer

    cfg = SDAConfig.from_yaml(_config_path(config))
    rank, world, local = setup_distributed()
    if world > 1 and device == "cuda":
        device = f"cuda:{local}"
    dev = _device(device)
    if jax_weights:
        from tornado_gcm_b200.model.jax_checkpoint_loader import load_jax_checkpoint

        gcm = load_jax_checkpoint(jax_weights, device=dev, resolution=cfg.model.resolution)
    else:
        gcm, _ = build_hybrid_gcm(cfg.model.resolution, dev, policy=cfg.policy, fixer=cfg.fixer)
    if not use_sda:
        cfg.scheduler.mode = "milestone"
        cfg.scheduler.check_interval = 10 ** 9
    dp = ("sharded" if parallel == "sharded" else True) if world > 1 else False
    trainer = SDATrainer(gcm, cfg, total_steps=steps, batch_size=batch_size, data_parallel=dp)
    if checkpoint and pathlib.Path(checkpoint).exists():
        logger.info("resuming from %s", checkpoint)
        trainer.load_checkpoint(checkpoint)
    hist = trainer.train(log_every=max(1, trainer.total_steps // 20))
    if hist and get_rank() == 0:
        click.echo(f"final loss {hist[-1]['loss']:.6g} after {hist[-1]['step']} steps")
    if checkpoint:
        trainer.save_checkpoint(checkpoint)
        if get_rank() == 0:
            logger.info("saved %s", checkpoint)


@main.command()
@click.option("--config", "-c", required=True)
@click.option("--checkpoint", "-k", required=True, type=click.Path(exists=True), help="Model checkpoint (.pt).")
@click.option("--input", "-i", "input_path", required=True, type=click.Path(exists=True),
              help="Initial condition (.pt or .npz of normalised pressure-level fields).")
@click.option("--output", "-o", "output_path", default="forecast.npz", show_default=True)
@click.option("--steps", "-s", default=40, show_default=True, help="6-hourly forecast steps.")
@click.option("--device", "-d", default="cuda", show_default=True)
@click.option("--use-sda/--no-sda", default=True, show_default=True)
def infer(config: str, checkpoint: str, input_path: str, output_path: str, steps: int, device: str,
          use_sda: bool) -> None:
    """Autoregressive forecast from an initial condition."""
    import torch

    from tornado_gcm_b200.inference.production import load_initial_condition, save_forecast
    from tornado_gcm_b200.precision.sda import SDAConfig

    cfg = SDAConfig.from_yaml(_config_path(config))
    dev = _device(device)
    sd = torch.load(checkpoint, map_location="cpu", weights_only=True)
    if use_sda:
        from tornado_gcm_b200.inference.sda_runner import SDAInference

        runner = SDAInference.from_state_dict(sd, cfg, device=dev, resolution=cfg.model.resolution)
    else:
        from tornado_gcm_b200.inference.runner import MPInference

        runner = MPInference.from_state_dict(sd, device=dev, resolution=cfg.model.resolution)
    ic = load_initial_condition(input_path, device=dev)
    forcings = ic.pop("forcings", None)
    traj = runner.rollout(ic, steps=steps, forcings=forcings, offload=True)
    save_forecast(traj, output_path)
    click.echo(f"wrote {len(traj)} steps to {output_path}")


@main.command()
@click.option("--config", "-c", required=True)
@click.option("--steps", "-s", default=2, show_default=True, help="Outer (6-h) steps per policy.")
@click.option("--device", "-d", default="cuda", show_default=True)
@click.option("--report", "-r", default="benchmark_report.txt", show_default=True)
def benchmark(config: str, steps: int, device: str, report: str) -> None:
    """Time one outer step per precision policy and report the drift against FP64 transforms."""
    from tornado_gcm_b200.precision.benchmarks import PrecisionBenchmark
    from tornado_gcm_b200.precision.sda import SDAConfig

    cfg = SDAConfig.from_yaml(_config_path(config))
    res = PrecisionBenchmark(sda_config=cfg, device=_device(device), n_steps=steps).run()
    text = res.report()
    click.echo(text)
    pathlib.Path(report).write_text(text, encoding="utf-8")


if __name__ == "__main__":
    main()
