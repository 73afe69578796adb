"""Model reference -> local path.

Parity: python/swiftllm/model_resolver.py:20-266 (local path, HF repo id,
HF URL with blob|resolve, ``org/repo:file`` GGUF selector,
``SWIFTLLM_MODEL_DIR`` and ``HF_TOKEN``). Downloads go through
``huggingface_hub`` when it is installed and the network allows; this build
is normally used offline with local paths or random-init presets.
"""

from __future__ import annotations

import os
import re
from pathlib import Path
from typing import Optional, Tuple

DEFAULT_MODEL_DIR = os.environ.get("SWIFTLLM_MODEL_DIR",
                                   os.path.join(Path.home(), ".cache", "swiftllm", "models"))

_HF_URL = re.compile(r"^https?://huggingface\.co/([^/]+/[^/]+)(?:/(?:blob|resolve)/[^/]+/(.+))?$")


def parse_model_ref(ref: str) -> Tuple[str, Optional[str], Optional[str]]:
    """Returns (kind, repo_or_path, filename); kind in {local, preset, hf}."""
    from .models.config import PRESETS
    if os.path.exists(ref):
        return "local", ref, None
    key = ref.lower()
    if key.startswith("dummy:") or key in PRESETS:
        return "preset", ref, None
    m = _HF_URL.match(ref)
    if m:
        return "hf", m.group(1), m.group(2)
    if ref.count("/") == 1 and ":" in ref:
        repo, fname = ref.split(":", 1)
        return "hf", repo, fname
    if re.match(r"^[\w.-]+/[\w.-]+$", ref):
        return "hf", ref, None
    return "local", ref, None


def resolve_model(model: str, download_dir: Optional[str] = None,
                  token: Optional[str] = None) -> str:
    kind, repo, fname = parse_model_ref(model)
    if kind in ("local", "preset"):
        return repo
    base = download_dir or DEFAULT_MODEL_DIR
    local = os.path.join(base, repo.replace("/", "--"))
    target = os.path.join(local, fname) if fname else local
    if os.path.exists(target):
        return target
    try:
        import huggingface_hub as hub  # type: ignore
    except ImportError as e:
        raise FileNotFoundError(
            f"{model!r} is not a local path or preset and huggingface_hub is not installed") from e
    tok = token or os.environ.get("HF_TOKEN")
    if fname:
        return hub.hf_hub_download(repo_id=repo, filename=fname, local_dir=local, token=tok)
    return hub.snapshot_download(repo_id=repo, local_dir=local, token=tok,
                                 allow_patterns=["*.json", "*.safetensors", "*.model", "*.txt"])


def list_local_models(base: Optional[str] = None):
    base = base or DEFAULT_MODEL_DIR
    if not os.path.isdir(base):
        return []
    return sorted(os.listdir(base))
