"""Alias of :mod:`femtotron_b200.models` under the reference's singular package name, with its
submodules (``femtotron_b200.model.llama``, ``.parallel_plan``, ``.model_loader``, ...) so that
code written against the reference's import paths resolves unchanged."""
import importlib
import sys

from femtotron_b200.models import *  # noqa: F401,F403
from femtotron_b200.models import __all__  # noqa: F401

for _sub in ("base", "layer_factory", "llama", "llama_causal", "llama_partial_model", "model_loader",
             "parallel_module_builder", "parallel_plan", "parallelize_model", "shard_loader", "layers",
             "materialize"):
    sys.modules[f"{__name__}.{_sub}"] = importlib.import_module(f"femtotron_b200.models.{_sub}")
del _sub
