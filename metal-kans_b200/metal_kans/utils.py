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


def build_train_step(model: Any, optimizer: Any, loss_fn: Any = None):
    """A training-step function for ``model`` (utils.py:70-124): the model's own fused
    ``train_step`` when it has one, else forward, the MSE gradient on the GPU, backward,
    ``optimizer.step()`` and ``zero_grad()``.  ``loss_fn`` is accepted and unused, like the
    reference (MSE is built in)."""
    lr = getattr(optimizer, "lr", 1e-3)
    b1 = getattr(optimizer, "beta1", 0.9)
    b2 = getattr(optimizer, "beta2", 0.999)
    eps = getattr(optimizer, "eps", 1e-8)
    wd = getattr(optimizer, "weight_decay", 0.01)

    if hasattr(model, "train_step"):
        def fused_step(x: np.ndarray, y: np.ndarray) -> float:
            return model.train_step(x, y, optimizer=optimizer, lr=lr, beta1=b1, beta2=b2, eps=eps,
                                    weight_decay=wd)
        return fused_step

    def standard_step(x: np.ndarray, y: np.ndarray) -> float:
        from . import _engine as E

        pred = np.ascontiguousarray(model(x), np.float32)
        t = np.ascontiguousarray(np.asarray(y, np.float32).reshape(pred.shape))
        diff = np.empty_like(pred)
        E.lib().metal_kan_calc_mse_loss_backward(pred.ctypes.data, t.ctypes.data, diff.ctypes.data,
                                                 pred.size, 2.0 / float(len(x)))
        model.backward(diff)
        optimizer.step()
        model.zero_grad()
        return 0.0

    return standard_step
