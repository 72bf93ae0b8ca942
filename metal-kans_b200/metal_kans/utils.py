"""Parameter counting and model size (``metal_kans/utils.py:10-67`` of the reference)."""
from __future__ import annotations

from typing import Any, Dict

import numpy as np

_COUNT_ATTRS = ("w_cheby", "w_rbf", "w_relu", "w_wav", "w_fourier", "w_jacobi", "w_p", "w_q",
                "w_spline", "w_up", "w_base", "bias", "translation", "scale")


def count_parameters(model: Any) -> int:
    """Total number of parameter elements of a layer or network."""
    if hasattr(model, "layers"):
        return sum(count_parameters(l) for l in model.layers)
    if hasattr(model, "gate_kan"):
        return sum(count_parameters(l) for l in (model.gate_kan, model.up_kan, model.down_kan))
    total = 0
    for attr in _COUNT_ATTRS:
        val = getattr(model, attr, None)
        if isinstance(val, np.ndarray):
            total += val.size
    return total


def get_model_size(model: Any) -> Dict[str, Any]:
    """Bytes, MB, element count and a summary string of the parameters."""
    total_bytes = 0
    total_params = 0
    subs = list(model.layers) if hasattr(model, "layers") else (
        [model.gate_kan, model.up_kan, model.down_kan] if hasattr(model, "gate_kan") else None)
    if subs is not None:
        for l in subs:
            s = get_model_size(l)
            total_bytes += s["bytes"]
            total_params += s["parameters"]
    else:
        for attr in _COUNT_ATTRS + ("weight_int8", "weight_int4"):
            val = getattr(model, attr, None)
            if isinstance(val, np.ndarray):
                total_bytes += val.nbytes
                total_params += val.size
    mb = total_bytes / (1024 * 1024)
    return {"bytes": total_bytes, "mb": mb, "parameters": total_params,
            "summary": f"{mb:.3f} MB ({total_bytes:,} bytes, {total_params:,} elements)"}
