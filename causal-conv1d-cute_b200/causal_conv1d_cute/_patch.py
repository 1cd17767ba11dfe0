"""Replace a module-level function everywhere it was imported by name (reference _patch.py:10-41).

``from package import function`` copies the function object into the importing module, so
patching only the defining module leaves those copies in place. wrap() therefore rebinds every
module attribute, across all loaded modules, that is the original function object.
"""

import functools
import importlib
import sys

_MARKER = "_causal_conv1d_cute"


def wrap(target, around):
    """Wrap the function at dotted path `target` with around(original, *args, **kwargs).

    Returns:
        How many module attributes now point at the wrapper; 0 when the function was already
        wrapped (calling wrap twice is a no-op).
    """
    module_name, _, name = target.rpartition(".")
    original = getattr(importlib.import_module(module_name), name)
    if getattr(original, _MARKER, False):
        return 0

    @functools.wraps(original)
    def wrapper(*args, **kwargs):
        return around(original, *args, **kwargs)

    setattr(wrapper, _MARKER, True)
    rebound = 0
    for module in list(sys.modules.values()):
        namespace = getattr(module, "__dict__", None)
        if not isinstance(namespace, dict):
            continue
        for attr in [a for a, v in list(namespace.items()) if v is original]:
            setattr(module, attr, wrapper)
            rebound += 1
    return rebound
