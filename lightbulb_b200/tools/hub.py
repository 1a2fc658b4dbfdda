"""Model sources: a local directory or a hub id ``org/name[@revision]`` resolved offline from the
Hugging Face cache layout.

Reference: ``src/hub.rs:13-221`` (``ModelSource`` local or hub id@revision, hf-hub downloads).
This box has no network, so a hub id is resolved from ``$HF_HUB_CACHE`` /
``$HF_HOME/hub`` / ``~/.cache/huggingface/hub`` (``models--org--name/snapshots/<commit>``, with
``refs/<revision>`` naming the commit); a missing snapshot is reported with the path searched.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import List, Optional


@dataclass
class ModelSource:
    kind: str                 # "local" | "hub"
    path_or_id: str
    revision: str = "main"

    @classmethod
    def parse(cls, s: str) -> "ModelSource":
        if os.path.exists(s) or s.startswith((".", "/", "~")):
            return cls("local", os.path.expanduser(s))
        rev = "main"
        if "@" in s:
            s, rev = s.split("@", 1)
        if s.count("/") != 1:
            raise ValueError(f"not a local path or an org/name hub id: {s!r}")
        return cls("hub", s, rev)


def cache_roots() -> List[str]:
    roots = []
    if os.environ.get("HF_HUB_CACHE"):
        roots.append(os.environ["HF_HUB_CACHE"])
    if os.environ.get("HF_HOME"):
        roots.append(os.path.join(os.environ["HF_HOME"], "hub"))
    roots.append(os.path.join(os.path.expanduser("~"), ".cache", "huggingface", "hub"))
    return roots


def resolve(source, roots: Optional[List[str]] = None) -> str:
    """Local directory of the model files."""
    src = ModelSource.parse(source) if isinstance(source, str) else source
    if src.kind == "local":
        if not os.path.isdir(src.path_or_id) and not os.path.isfile(src.path_or_id):
            raise FileNotFoundError(src.path_or_id)
        return src.path_or_id
    folder = "models--" + src.path_or_id.replace("/", "--")
    searched = []
    for root in roots or cache_roots():
        base = os.path.join(root, folder)
        searched.append(base)
        if not os.path.isdir(base):
            continue
        commit = src.revision
        ref = os.path.join(base, "refs", src.revision)
        if os.path.isfile(ref):
            with open(ref) as f:
                commit = f.read().strip()
        snap = os.path.join(base, "snapshots", commit)
        if os.path.isdir(snap):
            return snap
    raise FileNotFoundError(f"{src.path_or_id}@{src.revision} is not in the local hub cache "
                            f"(searched {searched}); downloads need network access")
