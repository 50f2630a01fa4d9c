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
        restored = adapter.load(target)
        expected = adapter.state_dict(model)
        actual = adapter.state_dict(restored)
        if set(actual) != set(expected):
            raise ValueError("Hugging Face export changed checkpoint tensor names")
        for name in sorted(expected):
            if not torch.equal(actual[name], expected[name]):
                raise ValueError(f"Hugging Face export failed exact reload verification: {name}")


def export_inference_bundle(model: torch.nn.Module, job: Any, directory: str | Path, *,
                            iteration: int | None) -> InferenceBundle:
    if iteration is None or iteration < 0:
        raise ValueError("export iteration must be non-negative")
    target = Path(directory).expanduser().resolve()
    if target.exists():
        raise FileExistsError(f"inference bundle already exists: {target}")
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


def load_inference_bundle(directory: str | Path):
    """Rebuild the model from ``job.json`` and load the digest-checked weights."""

    from representax_b200.config import JobConfig
    from representax_b200.train.job import load_model, prepare_model

    bundle = Path(directory).expanduser().resolve()
    manifest_path = bundle / "manifest.json"
    complete = bundle / COMPLETE_MARKER
    if not manifest_path.is_file() or not complete.is_file():
        raise FileNotFoundError(f"inference bundle is incomplete: {bundle}")
    manifest = json.loads(manifest_path.read_text())
    fingerprint = manifest.pop("fingerprint", None)
    if (manifest.get("schema_version") != EXPORT_SCHEMA or fingerprint != _fingerprint(manifest)
            or complete.read_text().strip() != fingerprint):
        raise ValueError(f"inference bundle manifest is invalid: {bundle}")
    model_path = bundle / manifest["native"]["model"]
    if _sha256(model_path) != manifest["native"]["model_sha256"]:
        raise ValueError(f"native model digest differs: {model_path}")
    job = JobConfig.model_validate_json((bundle / manifest["native"]["config"]).read_text())
    model = prepare_model(load_model(job), job)
    state = load_file(str(model_path))
    current = model.state_dict()
    missing = set(current) - set(state)
    unexpected = set(state) - set(current)
    if missing or unexpected:
        raise ValueError(f"native bundle does not match the model: missing={sorted(missing)[:5]}, "
                         f"unexpected={sorted(unexpected)[:5]}")
    model.load_state_dict({k: v.to(current[k].dtype) for k, v in state.items()})
    return model, job


__all__ = ["COMPLETE_MARKER", "EXPORT_SCHEMA", "InferenceBundle", "export_inference_bundle",
           "load_inference_bundle", "native_state_dict"]
