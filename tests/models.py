"""Session cache of seeded synthetic GGUF models (regenerated from seeds)."""
from __future__ import annotations

import hashlib
import os
import tempfile

import vxb_synth as S

_CACHE: dict[str, str] = {}
_DIR = tempfile.mkdtemp(prefix="vxb_models_")


def model_path(**kw) -> tuple[str, str]:
    """Returns (path, sha256) of make_model(**kw), written once per process."""
    key = repr(sorted(kw.items()))
    if key not in _CACHE:
        data = S.make_model(**kw)
        path = os.path.join(_DIR, hashlib.sha1(key.encode()).hexdigest() + ".gguf")
        with open(path, "wb") as f:
            f.write(data)
        _CACHE[key] = (path, hashlib.sha256(data).hexdigest())
    return _CACHE[key]
