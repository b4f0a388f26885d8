"""Load an export directory through the code it ships (reference homeimg_loader.py:13-48).

An export's model_index.json names its components as ("pipeline", class), and its root pipeline.py defines those
classes. ``load_homeimg_pipeline(root)`` executes that file (trusted code, as with a custom pipeline and
trust_remote_code) under a module name derived from the export's path and source, so two exports loaded in one
process never share classes; the bare name ``pipeline`` points at the module only while the pipeline loads and is
then restored to whatever it was before.

  from homeimg_loader import load_homeimg_pipeline
  pipe = load_homeimg_pipeline("exports/homeimg", device="cuda")
  out = pipe(["a red fox in the snow"], num_inference_steps=50, guidance_scale=3.0)
"""
import hashlib
import importlib.util
import json
import sys
import threading
from pathlib import Path

_LOCK = threading.RLock()


def export_module(root):
    """The export's pipeline.py as a module, imported once per (resolved path, source) pair."""
    root = Path(root).resolve()
    source = root / "pipeline.py"
    code = source.read_bytes()
    name = "_homeimg_export_" + hashlib.sha256(str(root).encode() + b"\0" + code).hexdigest()[:32]
    with _LOCK:
        mod = sys.modules.get(name)
        if mod is None:
            spec = importlib.util.spec_from_file_location(name, source)
            mod = importlib.util.module_from_spec(spec)
            sys.modules[name] = mod
            try:
                spec.loader.exec_module(mod)
            except BaseException:
                del sys.modules[name]
                raise
        return mod


def load_homeimg_pipeline(root, trust_remote_code=True, **kwargs):
    """Instantiate the pipeline class that model_index.json names, from the export's own pipeline.py."""
    if trust_remote_code is False:
        raise ValueError("a HomeIMG export is loaded by executing its pipeline.py: trust_remote_code must be True")
    root = Path(root).resolve()
    index = json.loads((root / "model_index.json").read_text())
    with _LOCK:
        mod = export_module(root)
        missing = object()
        before = sys.modules.get("pipeline", missing)
        sys.modules["pipeline"] = mod
        try:
            cls = getattr(mod, index["_class_name"])
            return cls.from_pretrained(str(root), **kwargs)
        finally:
            if before is missing:
                sys.modules.pop("pipeline", None)
            else:
                sys.modules["pipeline"] = before
