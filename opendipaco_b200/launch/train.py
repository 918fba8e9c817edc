"""``opendipaco train``: synchronous DiLoCo training on the GPUs of one node.

One process per GPU (``torchrun --nproc-per-node N -m opendipaco_b200.launch train
--config c.yaml``, or a single process for one GPU / the CPU): every rank builds the same
documents and shards from the config, owns a contiguous block of paths (or, with
``comm.dp > 1``, a path group shared by ``dp`` GPUs) and runs ``DiPaCoEngine.fit`` with
the backend chosen by the ``comm`` section:

* ``local``  -- one process holds every path;
* ``nccl``   -- torch.distributed NCCL all-reduce per module key (the baseline);
* ``nvlink`` -- the peer-memory outer step (reduce over sharers, Nesterov and write-back
  in our kernels), optionally with int4 or top-k outer payloads and intra-path data
  parallelism;
* ``auto``   -- ``local`` for one process, ``nvlink`` otherwise.

The ``kernels`` section selects the fused executor, CUDA-graph capture, the attention
kernels and the bound of cross-GPU waits. The reference drives the same training from
``examples/train_distributed.py``; this is its command-line counterpart.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch

from ..checkpoint import latest_checkpoint, load_checkpoint, save_checkpoint
from ..parallel.backend.local import LocalBackend
from ..train.loop import DiPaCoEngine, ExecOptions
from .config import LaunchConfig, dipaco_config, diloco_config


def _init_distributed(world: int, device: torch.device) -> None:
    import torch.distributed as dist

    if world > 1 and not dist.is_initialized():
        backend = "nccl" if device.type == "cuda" else "gloo"
        kw = {"device_id": device} if device.type == "cuda" else {}
        dist.init_process_group(backend, timeout=timedelta(seconds=300), **kw)


def make_backend(cfg: LaunchConfig, topology, world: int, device: torch.device):
    kind = cfg.comm.backend
    if kind == "auto":
        kind = "local" if world == 1 else ("nvlink" if device.type == "cuda" else "nccl")
    if kind == "local":
        if world != 1:
            raise ValueError("comm.backend: local needs a single process")
        return LocalBackend(topology)
    if kind == "nccl":
        from ..parallel.backend.torch_dist import TorchDistBackend

        return TorchDistBackend(topology, device=device, dp=cfg.comm.dp)
    if device.type != "cuda":
        raise ValueError("comm.backend: nvlink needs CUDA devices")
    from ..parallel.backend.nvlink import NVLinkBackend

    compress = None if cfg.comm.outer_compress == "none" else cfg.comm.outer_compress
    return NVLinkBackend(topology, device=device, dp=cfg.comm.dp, compress=compress, density=cfg.comm.outer_density)


def apply_kernel_options(cfg: LaunchConfig) -> ExecOptions:
    k = cfg.kernels
    if k.attention != "auto":
        os.environ["ODP_ATTN_IMPL"] = k.attention
    if torch.cuda.is_available():
        from ..ops._ext import available, ext

        if available():
            ext().set_peer_wait_ns(int(k.peer_wait_ms * 1e6))
    return ExecOptions(fused=k.fused, cuda_graphs=k.cuda_graphs)


def run_train(cfg: LaunchConfig, *, corpus=None, log_every: int = 1) -> list:
    """Train ``run.generations`` synchronous rounds; returns this rank's round metrics
    (rank 0 also writes the checkpoint when ``run.checkpoint_dir`` is set)."""
    world = int(os.environ.get("WORLD_SIZE", 1))
    rank, local = int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0))
    if cfg.run.device.startswith("cuda"):
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
    else:
        device = torch.device(cfg.run.device)
    _init_distributed(world, device)
    model, diloco = dipaco_config(cfg.model), diloco_config(cfg.diloco)
    if corpus is None:
        from .roles import build_corpus, build_documents

        corpus = build_corpus(cfg, model, build_documents(cfg))
    exec_opts = apply_kernel_options(cfg)
    backend = make_backend(cfg, model.build_topology(), world, device)
    engine = DiPaCoEngine(model, diloco, backend, device=device, seed=cfg.run.seed, exec_options=exec_opts)
    ckpt = cfg.run.checkpoint_dir
    if cfg.run.resume and ckpt and latest_checkpoint(ckpt):
        load_checkpoint(engine, latest_checkpoint(ckpt))
    done = engine._global_round
    history = engine.fit(corpus, max(0, cfg.run.generations - done), cfg.run.batch_size,
                         log_every=log_every if rank == 0 else 0, total_rounds=cfg.run.generations)
    if ckpt:
        save_checkpoint(engine, os.path.join(ckpt, f"round{engine._global_round:06d}"))
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        if hasattr(backend, "close"):
            backend.close()
    return history
