"""Atomic inference export bundles.

Parity: ``InferenceBundle``, ``export_inference_bundle`` and
``load_inference_bundle`` of src/representax/export.py:20-218: a
``final-model/`` directory written to a temporary sibling and published with
one ``os.replace``, holding ``native/job.json``, the native weights, an
optional verified Hugging Face checkpoint (``huggingface/``, LoRA merged,
exact reload check), ``manifest.json`` with a sha256 fingerprint and the
``REPRESENTAX_COMPLETE`` marker.

The native weights are ``native/model.safetensors`` keyed by the module's
parameter names (the reference writes an Equinox leaf file); loading
rebuilds the model from ``job.json`` and checks the digest.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import tempfile
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
from safetensors.torch import load_file, save_file

EXPORT_SCHEMA = "representax-inference-bundle-v1"
COMPLETE_MARKER = "REPRESENTAX_COMPLETE"


@dataclass(frozen=True)
class InferenceBundle:
    path: Path
    native_path: Path
    huggingface_path: Path | None
    iteration: int


def _sha256(path: Path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as handle:
        for block in iter(lambda: handle.read(1 << 22), b""):
            h.update(block)
    return h.hexdigest()


def _fingerprint(value: Any) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def _write_json(path: Path, value: Any) -> None:
    path.write_text(json.dumps(value, indent=2, sort_keys=True) + "\n")


def native_state_dict(model: torch.nn.Module) -> dict[str, torch.Tensor]:
    return {name: p.detach().float().cpu().contiguous() for name, p in model.state_dict().items()
            if torch.is_floating_point(p) or p.dtype in (torch.uint8, torch.int8, torch.uint16)}


def _export_huggingface(model, job, target: Path) -> None:
    from representax_b200.train.job import build_component

    config = job.export.huggingface
    adapter = build_component(config.adapter)
    from representax_b200.models.adapters import merge_quantized_lora

    model = merge_quantized_lora(model)
    source = Path(config.source_checkpoint).expanduser()
    if source.is_dir():
        shutil.copytree(source, target)
        for pattern in ("*.safetensors", "*.safetensors.index.json", "pytorch_model*.bin"):
            for stale in target.glob(pattern):
                stale.unlink()
    else:
        target.mkdir(parents=True)
    adapter.save(model, target)
    if config.verify_reload:
        _check_reload(adapter.state_dict(model), adapter.state_dict(adapter.load(target)), target)


def _check_reload(written: dict[str, torch.Tensor], reread: dict[str, torch.Tensor], where: Path) -> None:
    """The checkpoint read back from ``where`` has to equal what was written, bit for bit."""

    lost, gained = sorted(set(written) - set(reread)), sorted(set(reread) - set(written))
    differing = [name for name in sorted(set(written) & set(reread)) if not torch.equal(written[name], reread[name])]
    if lost or gained or differing:
        raise ValueError(f"the Hugging Face checkpoint at {where} does not read back as written: "
                         f"lost {lost[:3]}, gained {gained[:3]}, changed {differing[:3]}")


def export_inference_bundle(model: torch.nn.Module, job: Any, directory: str | Path, *,
                            iteration: int | None) -> InferenceBundle:
    if not (isinstance(iteration, int) and iteration >= 0):
        raise ValueError(f"export needs the iteration the weights come from (an int >= 0), got {iteration!r}")
    target = Path(directory).expanduser().resolve()
    if target.exists():
        raise FileExistsError(f"refusing to overwrite {target}: bundles are written once")
    target.parent.mkdir(parents=True, exist_ok=True)
    temporary = Path(tempfile.mkdtemp(prefix=f".{target.name}-", dir=target.parent)).resolve()
    try:
        native = temporary / "native"
        native.mkdir()
        (native / "job.json").write_text(job.model_dump_json(indent=2) + "\n")
        model_path = native / "model.safetensors"
        save_file(native_state_dict(model), str(model_path))
        hf_manifest = None
        if job.export.huggingface is not None:
            _export_huggingface(model, job, temporary / "huggingface")
            hf_manifest = {"directory": "huggingface", "verified": job.export.huggingface.verify_reload}
        manifest = {
            "schema_version": EXPORT_SCHEMA,
            "iteration": iteration,
            "selection": job.export.selection,
            "native": {"config": "native/job.json", "model": "native/model.safetensors",
                       "model_sha256": _sha256(model_path)},
            "huggingface": hf_manifest,
        }
        manifest["fingerprint"] = _fingerprint(manifest)
        _write_json(temporary / "manifest.json", manifest)
        (temporary / COMPLETE_MARKER).write_text(manifest["fingerprint"] + "\n")
        os.replace(temporary, target)
    except BaseException:
        shutil.rmtree(temporary, ignore_errors=True)
        raise
    return InferenceBundle(target, target / "native",
                           None if job.export.huggingface is None else target / "huggingface", iteration)


def _verified_manifest(bundle: Path) -> dict[str, Any]:
    """Read a bundle's manifest after checking marker, schema, fingerprint and weight digest."""

    try:
        manifest = json.loads((bundle / "manifest.json").read_text())
        marker = (bundle / COMPLETE_MARKER).read_text().strip()
    except FileNotFoundError as error:
        raise FileNotFoundError(f"{bundle} is not a finished bundle ({Path(error.filename).name} absent)") from None
    stated = manifest.pop("fingerprint", None)
    if manifest.get("schema_version") != EXPORT_SCHEMA:
        raise ValueError(f"{bundle}: schema {manifest.get('schema_version')!r}, expected {EXPORT_SCHEMA!r}")
    if not (stated == marker == _fingerprint(manifest)):
        raise ValueError(f"{bundle}: the manifest fingerprint, the marker and the manifest content disagree")
    weights = bundle / manifest["native"]["model"]
    if _sha256(weights) != manifest["native"]["model_sha256"]:
        raise ValueError(f"{weights} changed after export (sha256 differs from the manifest)")
    return manifest


def load_inference_bundle(directory: str | Path):
    """Rebuild the model from ``job.json`` and load the digest-checked weights."""

    from representax_b200.config import JobConfig
    from representax_b200.train.job import load_model, prepare_model

    bundle = Path(directory).expanduser().resolve()
    manifest = _verified_manifest(bundle)
    job = JobConfig.model_validate_json((bundle / manifest["native"]["config"]).read_text())
    model = prepare_model(load_model(job), job)
    model_path = bundle / manifest["native"]["model"]
    state = load_file(str(model_path))
    current = model.state_dict()
    if set(state) != set(current):
        raise ValueError(f"{model_path} holds other tensors than the model built from job.json: "
                         f"absent {sorted(set(current) - set(state))[:5]}, extra {sorted(set(state) - set(current))[:5]}")
    model.load_state_dict({k: v.to(current[k].dtype) for k, v in state.items()})
    return model, job


__all__ = ["COMPLETE_MARKER", "EXPORT_SCHEMA", "InferenceBundle", "export_inference_bundle",
           "load_inference_bundle", "native_state_dict"]
