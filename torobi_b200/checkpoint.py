"""Writing and restoring a QLoRA run's state.

The layout is the reference's (engine/src/checkpoint.rs:1-26, :160-200):

    <dir>/
    |-- manifest.json            what the checkpoint claims, checked on the way in
    |-- graph.json               the model description itself
    |-- parameters.safetensors   every parameter under its qualified path
    |-- optimizer.safetensors    m/<path> and v/<path> for the trained ones
    `-- random.safetensors       the RNG key (from the seed)

It is laid out in ``<dir>.writing``, read back and checked against the
manifest, and only then renamed into place (a previous checkpoint is moved
aside first and dropped last), so an interrupted write leaves no
half-checkpoint (:145-230).  Restoring checks the config digest, the
optimizer, and every parameter's path, shape and dtype before touching the
run (:310-400); a mismatch is refused, not absorbed.

The parameters are the run's: the quantized base as MLX's three tensors per
linear (``.weight`` u32 codes, ``.scales``, ``.biases``), norms, embedding and
head in bf16, and the adapters' f32 master matrices (the only trained ones).
"""
from __future__ import annotations

import hashlib
import json
import os
import platform as _platform
import shutil
from dataclasses import asdict
from pathlib import Path

import torch

from .weights import adapter_paths, dtype_spelling, linear_path

SCHEMA_VERSION = 2
SEMANTICS_VERSION = 1
GRAPH_FILE = "graph.json"


def graph_json(cfg) -> str:
    """The model description, canonical JSON (sorted keys)."""
    return json.dumps(asdict(cfg), sort_keys=True)


def config_digest(cfg) -> str:
    return hashlib.sha256(graph_json(cfg).encode()).hexdigest()


def optimizer_config(opt) -> dict:
    """The rule, as the reference serialises it (engine/src/optimizer.rs:16-44)."""
    return {"kind": "adamw", "lr": float(opt.lr), "beta1": float(opt.beta1),
            "beta2": float(opt.beta2), "eps": float(opt.eps),
            "weight_decay": float(opt.weight_decay),
            "clip": None if opt.clip is None else float(opt.clip)}


def run_parameters(model) -> list[tuple[str, torch.Tensor, bool]]:
    """(qualified path, tensor, trained) for every parameter of the run, in
    declaration order."""
    out = [("model.embed_tokens.weight", model.embed, False)]
    for li, blk in enumerate(model.blocks):
        out.append((f"model.layers.{li}.input_layernorm.weight", blk.input_norm, False))
        for name, w in blk.linears.items():
            if name == "gate_proj":
                out.append((f"model.layers.{li}.post_attention_layernorm.weight", blk.post_norm,
                            False))
            path = linear_path(li, name)
            out.append((f"{path}.weight", w.codes, False))
            out.append((f"{path}.scales", w.scales, False))
            out.append((f"{path}.biases", w.biases, False))
            if w.bias is not None:
                out.append((f"{path}.bias", w.bias, False))
            ad = blk.adapters.get(name)
            if ad is not None:
                pa, pb = adapter_paths(li, name)
                out.append((pa, ad.a, True))
                out.append((pb, ad.b, True))
    out.append(("model.norm.weight", model.final_norm, False))
    if model.lm_head is not None:
        out.append(("lm_head.weight", model.lm_head, False))
    return out


def _slots(model) -> dict[str, tuple[torch.Tensor, torch.Tensor]]:
    """AdamW moments by trained path: views into the store's flat m and v."""
    st = model.store
    out = {}
    for li, blk in enumerate(model.blocks):
        for name, ad in blk.adapters.items():
            if ad is None:
                continue
            pa, pb = adapter_paths(li, name)
            for path, view in ((pa, ad.a), (pb, ad.b)):
                off = view.storage_offset() - st.params.storage_offset()
                n = view.numel()
                out[path] = (st.m[off:off + n].view(view.shape), st.v[off:off + n].view(view.shape))
    return out


def _rng_key(seed: int) -> torch.Tensor:
    return torch.tensor([(seed >> 32) & 0xFFFFFFFF, seed & 0xFFFFFFFF], dtype=torch.uint32)


def _save(tensors: dict[str, torch.Tensor], path: Path) -> None:
    from safetensors.torch import save_file

    save_file({k: v.detach().to("cpu", copy=True).contiguous() for k, v in tensors.items()},
              str(path))


def _load(path: Path) -> dict[str, torch.Tensor]:
    from safetensors.torch import load_file

    return load_file(str(path))


def manifest_of(trainer, seed: int, step: int, run) -> dict:
    params = []
    for path, t, trained in run_parameters(trainer.model):
        spelled = dtype_spelling(t.dtype)
        if spelled is None:
            raise ValueError(f"parameter {path!r} holds {t.dtype}, which the dtype vocabulary "
                             "cannot name; a checkpoint that recorded it could not be read back")
        params.append({"path": path, "shape": list(t.shape), "dtype": spelled,
                       "trained": trained})
    return {
        "schema_version": SCHEMA_VERSION,
        "config_digest": config_digest(trainer.model.cfg),
        "semantics_version": SEMANTICS_VERSION,
        "step": int(step),
        "optimizer": optimizer_config(trainer.opt),
        "optimizer_steps": int(trainer.t),
        "seed": int(seed),
        "parameters": params,
        "build": {"package": "torobi_b200"},
        "platform": {"os": _platform.system().lower(), "arch": _platform.machine()},
        "run": run if run is not None else {},
    }


def _lay_out(staging: Path, trainer, seed: int, step: int, run) -> None:
    model = trainer.model
    (staging / GRAPH_FILE).write_text(graph_json(model.cfg))
    _save({p: t for p, t, _ in run_parameters(model)}, staging / "parameters.safetensors")
    slots = _slots(model)
    named = {}
    for path, (m, v) in slots.items():
        named[f"m/{path}"] = m
        named[f"v/{path}"] = v
    _save(named, staging / "optimizer.safetensors")
    _save({"key": _rng_key(seed)}, staging / "random.safetensors")
    (staging / "manifest.json").write_text(
        json.dumps(manifest_of(trainer, seed, step, run), indent=2))


def _sync_dir(d: Path) -> None:
    fd = os.open(str(d), os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def save(trainer, directory, seed: int = 0, step: int | None = None, run=None) -> Path:
    """Writes the run's state to ``directory`` atomically; returns it.

    Everything on the device is synchronised first (the tensors are copied
    to the host), and the trainer's last step is settled, so a step whose
    gradient norm was not finite (skipped on the device) is not counted in
    the optimizer step count the checkpoint records."""
    trainer.settle()
    d = Path(directory)
    staging = d.with_name(d.name + ".writing")
    if staging.exists():
        shutil.rmtree(staging)
    staging.mkdir(parents=True)
    _lay_out(staging, trainer, seed, trainer.steps if step is None else step, run)
    # Nothing takes the name before it reads back.
    try:
        read(staging)
    except Exception as e:  # noqa: BLE001
        raise RuntimeError(f"the checkpoint just written does not read back: {e}") from e
    for f in staging.iterdir():
        fd = os.open(str(f), os.O_RDONLY)
        try:
            os.fsync(fd)
        finally:
            os.close(fd)
    _sync_dir(staging)
    displaced = None
    if d.exists():
        displaced = d.with_name(d.name + ".replaced")
        if displaced.exists():
            shutil.rmtree(displaced)
        d.rename(displaced)
    staging.rename(d)
    if displaced is not None:
        shutil.rmtree(displaced, ignore_errors=True)
    _sync_dir(d.parent if str(d.parent) else Path("."))
    return d


def read_manifest(directory) -> dict:
    m = json.loads((Path(directory) / "manifest.json").read_text())
    if m.get("schema_version") != SCHEMA_VERSION:
        raise ValueError(f"checkpoint schema {m.get('schema_version')} is not {SCHEMA_VERSION}")
    return m


def read(directory) -> dict:
    """Reads a checkpoint and checks it against its own manifest: every
    parameter present with the recorded shape and dtype, the moments of every
    trained one, the description's digest.  Returns the loaded tensors."""
    d = Path(directory)
    manifest = read_manifest(d)
    graph = (d / GRAPH_FILE).read_text()
    if hashlib.sha256(graph.encode()).hexdigest() != manifest["config_digest"]:
        raise ValueError("graph.json does not match the manifest's config digest")
    params = _load(d / "parameters.safetensors")
    for e in manifest["parameters"]:
        t = params.get(e["path"])
        if t is None:
            raise ValueError(f"the checkpoint has no parameter {e['path']!r}")
        if list(t.shape) != list(e["shape"]) or dtype_spelling(t.dtype) != e["dtype"]:
            raise ValueError(f"parameter {e['path']!r} is {dtype_spelling(t.dtype)} "
                             f"{list(t.shape)}, the manifest says {e['dtype']} {e['shape']}")
    if len(params) != len(manifest["parameters"]):
        raise ValueError(f"parameters.safetensors holds {len(params)} tensors, the manifest "
                         f"names {len(manifest['parameters'])}")
    opt = _load(d / "optimizer.safetensors")
    for e in manifest["parameters"]:
        if e["trained"]:
            for k in (f"m/{e['path']}", f"v/{e['path']}"):
                t = opt.get(k)
                if t is None or list(t.shape) != list(e["shape"]):
                    raise ValueError(f"the checkpoint has no optimizer state {k!r} of shape "
                                     f"{e['shape']}")
    rng = _load(d / "random.safetensors")
    if "key" not in rng:
        raise ValueError("the checkpoint has no RNG state")
    return {"manifest": manifest, "parameters": params, "optimizer": opt, "rng": rng["key"]}


def restore(trainer, directory) -> dict:
    """Checks a checkpoint against the run and, only if all of it belongs,
    copies it in: every parameter, the AdamW moments and step count.
    Returns the manifest."""
    loaded = read(directory)
    m = loaded["manifest"]
    model = trainer.model
    digest = config_digest(model.cfg)
    if m["config_digest"] != digest:
        raise ValueError(f"this checkpoint belongs to another model (digest "
                         f"{m['config_digest'][:12]}, not {digest[:12]})")
    if m["optimizer"] != optimizer_config(trainer.opt):
        raise ValueError(f"this checkpoint was written by a different optimizer "
                         f"({m['optimizer']})")
    mine = run_parameters(model)
    if len(m["parameters"]) != len(mine):
        raise ValueError(f"this checkpoint has {len(m['parameters'])} parameters, this run "
                         f"has {len(mine)}")
    for i, ((path, t, trained), e) in enumerate(zip(mine, m["parameters"])):
        if e["path"] != path:
            raise ValueError(f"parameter {i} is {path!r} here and {e['path']!r} in the "
                             "checkpoint")
        got = loaded["parameters"][path]
        if tuple(got.shape) != tuple(t.shape) or got.dtype != t.dtype:
            raise ValueError(f"parameter {path!r}: checkpoint {got.dtype} {tuple(got.shape)} is "
                             f"not {t.dtype} {tuple(t.shape)}")
        if e["trained"] != trained:
            raise ValueError(f"parameter {path!r} is trained in one and frozen in the other")
    # Every check passed: commit.
    for path, t, _ in mine:
        t.copy_(loaded["parameters"][path].to(t.device))
    for path, (mm, vv) in _slots(model).items():
        mm.copy_(loaded["optimizer"][f"m/{path}"].to(mm.device))
        vv.copy_(loaded["optimizer"][f"v/{path}"].to(vv.device))
    model.store.refresh_bf16(full=True)
    trainer.t = int(m["optimizer_steps"])
    trainer.steps = int(m["step"])
    return m
