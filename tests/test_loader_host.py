"""A Qwen3-MoE checkpoint loaded into the drop-in ``MoE`` by the reference's own loader
(prism_infer/utils/loader.py:63-88, ``load_model``), single rank and expert parallel.

A tiny safetensors checkpoint is written with the reference's weight names
(``model.layers.{i}.mlp.gate.weight``, ``...mlp.experts.{e}.gate_proj/up_proj/down_proj.weight``;
gate_proj and up_proj are packed into ``gate_up_proj`` by ``packed_modules_mapping``,
prism_infer/models/qwen3.py:214-220). ``load_model`` then writes them through the
``weight_loader``s of the module's per-expert views into the stacked expert storage. Under expert
parallelism (two gloo ranks) ``_remap_expert_weight`` (loader.py:27-60) keeps each rank's
experts, mapped to ``ep_moe.local_experts.{le}``, and skips the others. No GPU: loading is host
work. The loader is imported from the reference's source tree, so the test is skipped where that
tree is absent.
"""
import os
import socket
import sys
import tempfile
from pathlib import Path

import pytest
import torch
from torch import nn

REF = Path(os.environ.get("PRISM_REFERENCE", "/root/reference"))
pytestmark = pytest.mark.skipif(not (REF / "prism_infer" / "utils" / "loader.py").exists(),
                                reason="the reference's source tree is not available")
H, I, E, k, LAYERS = 32, 16, 8, 2, 2


def write_checkpoint(path: Path, seed: int = 0) -> dict:
    from safetensors.torch import save_file
    g = torch.Generator().manual_seed(seed)
    tensors = {}
    for li in range(LAYERS):
        p = f"model.layers.{li}.mlp"
        tensors[f"{p}.gate.weight"] = torch.randn(E, H, generator=g)
        for e in range(E):
            tensors[f"{p}.experts.{e}.gate_proj.weight"] = torch.randn(I, H, generator=g)
            tensors[f"{p}.experts.{e}.up_proj.weight"] = torch.randn(I, H, generator=g)
            tensors[f"{p}.experts.{e}.down_proj.weight"] = torch.randn(H, I, generator=g)
    save_file(tensors, str(path / "model.safetensors"))
    return tensors


def build_model():
    from prism_infer_b200.layers.moe import MoE

    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.mlp = MoE(H, I, E, k)

    class Model(nn.Module):
        packed_modules_mapping = {"gate_proj": ("gate_up_proj", 0),
                                  "up_proj": ("gate_up_proj", 1)}

        def __init__(self):
            super().__init__()
            self.model = nn.Module()
            self.model.layers = nn.ModuleList(Layer() for _ in range(LAYERS))

    return Model()


def check_loaded(model, tensors, rank, W):
    El = E // W
    for li, layer in enumerate(model.model.layers):
        p = f"model.layers.{li}.mlp"
        moe = layer.mlp
        assert torch.equal(moe.gate.weight, tensors[f"{p}.gate.weight"])
        bank = moe.ep_moe if W > 1 else moe
        for le in range(El):
            e = rank * El + le
            assert torch.equal(bank.w_gate_up[le, :I], tensors[f"{p}.experts.{e}.gate_proj.weight"])
            assert torch.equal(bank.w_gate_up[le, I:], tensors[f"{p}.experts.{e}.up_proj.weight"])
            assert torch.equal(bank.w_down[le], tensors[f"{p}.experts.{e}.down_proj.weight"])


def _import_loader():
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from prism_infer.utils.loader import load_model
    return load_model


def test_single_rank_checkpoint_loads_into_stacked_storage():
    from prism_infer_b200.engine.parallel import set_expert_parallel_size
    load_model = _import_loader()
    set_expert_parallel_size(1)
    with tempfile.TemporaryDirectory() as d:
        tensors = write_checkpoint(Path(d))
        model = build_model()
        for layer in model.model.layers:          # stale values must be overwritten
            layer.mlp.w_gate_up.fill_(7.0)
            layer.mlp.w_down.fill_(7.0)
        load_model(model, d)
    check_loaded(model, tensors, 0, 1)


def _ep_worker(rank, W, port, ckpt, outdir):
    import torch.distributed as dist
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=W)
    from prism_infer_b200.engine.parallel import set_expert_parallel_size
    load_model = _import_loader()
    set_expert_parallel_size(W)
    model = build_model()
    load_model(model, ckpt)
    from safetensors.torch import load_file
    check_loaded(model, load_file(str(Path(ckpt) / "model.safetensors")), rank, W)
    names = set(dict(model.named_parameters()))
    assert f"model.layers.0.mlp.ep_moe.local_experts.{E // W - 1}.down_proj.weight" in names
    Path(outdir, f"ok{rank}").write_text("ok")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("W", [2, 4])
def test_expert_parallel_checkpoint_keeps_each_ranks_experts(W):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d, tempfile.TemporaryDirectory() as out:
        write_checkpoint(Path(d), seed=W)
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        mp.start_processes(_ep_worker, args=(W, port, d, out), nprocs=W, join=True,
                           start_method="spawn")
        assert sorted(os.listdir(out)) == [f"ok{r}" for r in range(W)]
