"""Model snapshots: manifest-bound integrity and diffusers/safetensors weight loading.

``verify_snapshot(dir, manifest)`` hashes every file a manifest lists ({relative path:
sha256}) and rejects missing, extra or altered files before anything is loaded.
``load_diffusers_transformer(model, dir)`` reads the diffusers layout
(``transformer/diffusion_pytorch_model*.safetensors`` with an optional index json)
into one of our modules, whose parameter names follow diffusers, and rebuilds the
fused weights.  Reference: workers/ditserve/runtime/model_integrity.py:19-66.
"""
from __future__ import annotations

import json
from pathlib import Path

from . import file_hash


class IntegrityError(RuntimeError):
    pass


def build_manifest(root) -> dict:
    root = Path(root)
    return {str(p.relative_to(root)): file_hash(p) for p in sorted(root.rglob("*")) if p.is_file()}


def verify_snapshot(root, manifest: dict, allow_extra: bool = False) -> dict:
    root = Path(root)
    if not root.is_dir():
        raise IntegrityError(f"snapshot directory {root} is missing")
    present = {str(p.relative_to(root)) for p in root.rglob("*") if p.is_file()}
    missing = sorted(set(manifest) - present)
    extra = sorted(present - set(manifest))
    if missing:
        raise IntegrityError(f"snapshot is missing {missing[:5]}")
    if extra and not allow_extra:
        raise IntegrityError(f"snapshot has unexpected files {extra[:5]}")
    for rel, digest in manifest.items():
        if file_hash(root / rel) != digest:
            raise IntegrityError(f"{rel} does not match its manifest hash")
    return dict(verified=True, files=len(manifest))


def load_diffusers_transformer(model, root, subfolder: str = "transformer", strict: bool = True):
    from safetensors.torch import load_file
    d = Path(root) / subfolder if subfolder else Path(root)
    index = d / "diffusion_pytorch_model.safetensors.index.json"
    if index.exists():
        files = sorted(set(json.loads(index.read_text())["weight_map"].values()))
    else:
        files = ["diffusion_pytorch_model.safetensors"]
    state = {}
    for f in files:
        state.update(load_file(str(d / f)))
    own = model.state_dict()
    converted = {k: v.to(own[k].dtype) if k in own else v for k, v in state.items()}
    missing, unexpected = model.load_state_dict(converted, strict=False)
    missing = [m for m in missing if not m.startswith("pos_embed.pos_embed")]
    if strict and (missing or unexpected):
        raise IntegrityError(f"checkpoint mismatch: missing {missing[:5]}, unexpected {unexpected[:5]}")
    model.prepare()
    return dict(files=len(files), tensors=len(state), missing=missing, unexpected=list(unexpected))
