"""Drop-in ``KernelGenerator``: the reference's per-op lowering interface.

``tensorlang/compiler.py`` lowers each ``let`` by calling one method of
``tensorlang/kernel_generator.py``'s ``KernelGenerator`` and keeps the
returned ``(cuda_source, kernel_info)``; ``kernel_info[0]`` is the dispatch
key of ``TensorCompiler._execute_single_kernel`` (compiler.py:365-673).

This class has the same method names, argument lists and ``kernel_info``
tuples (checked against the reference generator in
``tests/test_cpu_boundary.py``).  The source string is empty: the kernels
are the prebuilt sm_100a kernels of libtlb200 and the fused elementwise
regions the backend generates itself, so nothing per-op needs compiling.

Differences, all additions:

* ``gelu`` and ``swish`` exist (the reference has grammar and type rules but
  no generator method);
* ``cross_entropy`` accepts one-hot targets ``(B, C)`` ->
  ``('cross_entropy_onehot', ...)``;
* ``argmax``/``argmin`` accept axis 0 (``'argmax_axis0'``, ``'argmin_axis0'``)
  and ``argmin`` the full tensor (``'argmin_full'``);
* shapes the reference returns ``None`` for raise ``NotImplementedError``;
* ``numpy_broadcast=True`` (the backend's ``semantics="numpy"``) gives a
  square 2-D op 1-D the NumPy kernel (``B[j]``) instead of the per-row one.
"""
from __future__ import annotations

import numpy as np

_OPS4 = ("add", "minus", "mult", "div")

_SIGNATURES = {
    "elementwise": _OPS4, "binary_broadcast": _OPS4, "binary_1d_broadcast": _OPS4,
    "binary_general_broadcast": _OPS4, "fill": ("fill",), "matmul": ("matmul",),
    "relu": ("relu",), "sigmoid": ("sigmoid",), "tanh": ("tanh",), "gelu": ("gelu",),
    "swish": ("swish",), "softmax": ("softmax",), "greater_broadcast": ("greater",),
    "less_broadcast": ("less",), "equal": ("equal",), "sum": ("sum",), "mean": ("mean",),
    "slice": ("slice",), "max": ("max",), "min": ("min",), "argmax": ("argmax",),
    "argmin": ("argmin",), "linear": ("linear",), "layer_norm": ("layer_norm",),
    "concat": ("concat",), "reshape": ("reshape",), "instance_norm": ("instance_norm",),
    "batch_norm": ("batch_norm",), "transpose": ("transpose",), "mse_loss": ("mse_loss",),
    "cross_entropy": ("cross_entropy",),
}


def _prod(shape) -> int:
    return int(np.prod([int(d) for d in shape])) if len(shape) else 1


class KernelGenerator:
    """Per-op lowering with the reference's signatures (kernel_generator.py:9-2132)."""

    def __init__(self, DEBUG_MODE=False, numpy_broadcast=False):
        self.DEBUG_MODE = DEBUG_MODE
        self.numpy_broadcast = numpy_broadcast

    def _validate(self, kernel_type, op_type):
        """kernel_generator.py:21-146: unknown kernel types / ops raise ValueError."""
        if kernel_type not in _SIGNATURES:
            raise ValueError(f"Generator: Unsupported kernel type: {kernel_type}")
        if op_type not in _SIGNATURES[kernel_type]:
            raise ValueError(f"Unsupported operation for {kernel_type}: {op_type}")

    def cuda_header(self):
        return "// TensorLang program lowered to libtlb200 (sm_100a)\n"

    def cuda_debug(self):
        return ""

    # -- elementwise -----------------------------------------------------------
    def elementwise(self, op_type, name, arg1, arg2, size):
        self._validate("elementwise", op_type)
        return "", (op_type, name, arg1, arg2, size)

    def binary_broadcast(self, op_name, op_type, name, arg1, arg2, shape1, shape2, output_shape):
        self._validate("binary_broadcast", op_type)
        rows, cols = output_shape
        # the reference's rule (:303-348): B[i] whenever the row counts match;
        # NumPy's reads B[j] when the columns match too (square inputs)
        square = self.numpy_broadcast and shape1[1] == shape2[0]
        if shape1[0] == shape2[0] and not square:
            return "", (f"{op_type}_broadcast_rows", name, arg1, arg2, rows, cols)
        return "", (f"{op_type}_broadcast", name, arg1, arg2, rows, cols)

    def binary_1d_broadcast(self, op_type, name, arg1, arg2, size):
        self._validate("binary_1d_broadcast", op_type)
        return "", (f"{op_type}_scalar", name, arg1, arg2, size)

    def binary_general_broadcast(self, op_type, name, arg1, arg2, shape1, shape2, output_shape):
        self._validate("binary_general_broadcast", op_type)
        nd = len(output_shape)
        total = _prod(output_shape)
        p1 = (1,) * (nd - len(shape1)) + tuple(shape1)
        p2 = (1,) * (nd - len(shape2)) + tuple(shape2)
        return "", ("general_broadcast", op_type, name, arg1, arg2, p1, p2, output_shape, total)

    def fill(self, op_type, name, arg1, arg2, size, op_value):
        self._validate("fill", op_type)
        return "", (op_type, name, arg1, arg2, size, op_value)

    def generate_unary_op_kernel(self, op_type, name, arg1, size, operation=None):
        return "", (op_type, name, arg1, None, size)

    def relu(self, op_type, name, arg1, size):
        self._validate("relu", op_type)
        return self.generate_unary_op_kernel(op_type, name, arg1, size)

    def sigmoid(self, op_type, name, arg1, size):
        self._validate("sigmoid", op_type)
        return self.generate_unary_op_kernel(op_type, name, arg1, size)

    def tanh(self, op_type, name, arg1, size):
        self._validate("tanh", op_type)
        return self.generate_unary_op_kernel(op_type, name, arg1, size)

    def gelu(self, op_type, name, arg1, size):
        self._validate("gelu", op_type)
        return self.generate_unary_op_kernel(op_type, name, arg1, size)

    def swish(self, op_type, name, arg1, size):
        self._validate("swish", op_type)
        return self.generate_unary_op_kernel(op_type, name, arg1, size)

    def greater_broadcast(self, op_type, name, arg1, arg2, shape1, shape2, output_shape, size):
        if tuple(shape1) == tuple(shape2):
            return "", (op_type, name, arg1, arg2, size)
        rows, cols = output_shape
        return "", (f"{op_type}_broadcast", name, arg1, arg2, rows, cols)

    def less_broadcast(self, op_type, name, arg1, arg2, shape1, shape2, output_shape):
        if tuple(shape1) == tuple(shape2):
            return "", (f"{op_type}", name, arg1, arg2, _prod(output_shape))
        rows, cols = output_shape
        return "", (f"{op_type}_broadcast", name, arg1, arg2, rows, cols)

    def equal(self, op_type, name, arg1, arg2, shape1, shape2, output_shape):
        if tuple(shape1) == tuple(shape2):
            return "", (f"{op_type}", name, arg1, arg2, _prod(output_shape))
        rows, cols = output_shape
        return "", (f"{op_type}", name, arg1, arg2, rows, cols)

    # -- matmul / linear -------------------------------------------------------
    def matmul(self, op_type, name, arg1, arg2, m, n, p):
        self._validate("matmul", op_type)
        return "", (op_type, name, arg1, arg2, m, n, p)

    def linear(self, op_type, name, input_name, weight_name, bias_name, input_shape,
               weight_shape, output_shape):
        if len(input_shape) == 1:
            return "", (f"{op_type}_1d", name, input_name, weight_name, bias_name,
                        int(input_shape[0]), int(output_shape[0]))
        if len(input_shape) == 2:
            return "", (f"{op_type}_2d", name, input_name, weight_name, bias_name,
                        int(input_shape[0]), int(input_shape[1]), int(output_shape[1]))
        raise NotImplementedError(f"linear on input shape {tuple(input_shape)}")

    # -- softmax / norms -------------------------------------------------------
    def softmax(self, op_type, name, tensor_name, input_shape, axis):
        self._validate("softmax", op_type)
        if axis is None:
            axis = len(input_shape) - 1
        if len(input_shape) == 2 and axis == 1:
            return "", ("softmax", name, tensor_name, None, int(input_shape[0]),
                        int(input_shape[1]), axis)
        if len(input_shape) == 1:
            return "", ("softmax_1d", name, tensor_name, None, int(input_shape[0]))
        raise NotImplementedError(f"softmax of shape {tuple(input_shape)} along axis {axis}")

    def layer_norm(self, op_type, name, tensor_name, axis, eps, input_shape):
        if axis is None:
            axis = len(input_shape) - 1
        if len(input_shape) == 2:
            rows, cols = int(input_shape[0]), int(input_shape[1])
            if axis == 1:
                return "", (f"{op_type}_2d", name, tensor_name, None, rows, cols, eps)
            if axis == 0:
                return "", (f"{op_type}_axis0", name, tensor_name, None, rows, cols, eps)
        elif len(input_shape) == 1:
            return "", (f"{op_type}_1d", name, tensor_name, None, int(input_shape[0]), eps)
        raise NotImplementedError(f"layer_norm of shape {tuple(input_shape)} along axis {axis}")

    def batch_norm(self, op_type, name, input_shape, tensor_name, running_mean_name, eps,
                   running_var_name):
        if len(input_shape) == 2:
            return "", (f"{op_type}_2d", name, tensor_name, running_mean_name,
                        int(input_shape[0]), int(input_shape[1]), eps, running_var_name)
        raise NotImplementedError(f"batch_norm of shape {tuple(input_shape)}")

    def instance_norm(self, op_type, name, tensor_name, input_shape, eps):
        if len(input_shape) == 2:
            return "", (f"{op_type}_2d", name, tensor_name, None, None,
                        int(input_shape[0]), int(input_shape[1]), eps)
        raise NotImplementedError(f"instance_norm of shape {tuple(input_shape)}")

    # -- reductions -----------------------------------------------------------
    def _reduce(self, op_type, name, tensor_name, axis, input_shape):
        if axis is None:
            return "", (f"{op_type}_full", name, tensor_name, None, _prod(input_shape))
        if len(input_shape) == 2 and axis == 1:
            return "", (f"{op_type}_axis", name, tensor_name, None, int(input_shape[0]),
                        int(input_shape[1]), axis)
        if len(input_shape) == 2 and axis == 0:
            return "", (f"{op_type}_axis0", name, tensor_name, None, int(input_shape[0]),
                        int(input_shape[1]), axis)
        raise NotImplementedError(f"{op_type} of shape {tuple(input_shape)} along axis {axis}")

    def sum(self, op_type, name, tensor_name, axis, input_shape):
        return self._reduce(op_type, name, tensor_name, axis, input_shape)

    def mean(self, op_type, name, tensor_name, axis, input_shape):
        return self._reduce(op_type, name, tensor_name, axis, input_shape)

    def max(self, op_type, name, tensor_name, axis, input_shape):
        return self._reduce(op_type, name, tensor_name, axis, input_shape)

    def min(self, op_type, name, tensor_name, axis, input_shape):
        return self._reduce(op_type, name, tensor_name, axis, input_shape)

    def argmax(self, op_type, name, tensor_name, axis, input_shape):
        if axis is None:
            # the reference tags the full argmax 'argmax_axis' with one dim
            return "", (f"{op_type}_axis", name, tensor_name, None, _prod(input_shape))
        if len(input_shape) == 2 and axis == 1:
            return "", (f"{op_type}_axis", name, tensor_name, None, int(input_shape[0]),
                        int(input_shape[1]), axis)
        if len(input_shape) == 2 and axis == 0:
            return "", (f"{op_type}_axis0", name, tensor_name, None, int(input_shape[0]),
                        int(input_shape[1]), axis)
        raise NotImplementedError(f"argmax of shape {tuple(input_shape)} along axis {axis}")

    def argmin(self, op_type, name, tensor_name, axis, input_shape):
        if axis is None:
            return "", (f"{op_type}_full", name, tensor_name, None, _prod(input_shape))
        if len(input_shape) == 2 and axis == 1:
            return "", (f"{op_type}_axis", name, tensor_name, None, int(input_shape[0]),
                        int(input_shape[1]), axis)
        if len(input_shape) == 2 and axis == 0:
            return "", (f"{op_type}_axis0", name, tensor_name, None, int(input_shape[0]),
                        int(input_shape[1]), axis)
        raise NotImplementedError(f"argmin of shape {tuple(input_shape)} along axis {axis}")

    # -- losses ------------------------------------------------------------------
    def cross_entropy(self, op_type, name, pred_name, pred_shape, target_shape, target_name):
        if len(pred_shape) == 2 and len(target_shape) == 1:
            return "", (f"{op_type}", name, pred_name, target_name, int(pred_shape[0]),
                        int(pred_shape[1]))
        if len(pred_shape) == 2 and tuple(target_shape) == tuple(pred_shape):
            return "", (f"{op_type}_onehot", name, pred_name, target_name, int(pred_shape[0]),
                        int(pred_shape[1]))
        raise NotImplementedError(f"cross_entropy of {tuple(pred_shape)} vs {tuple(target_shape)}")

    def mse_loss(self, op_type, name, pred_name, target_name, total_elements):
        return "", (f"{op_type}", name, pred_name, target_name, total_elements)

    # -- data movement ---------------------------------------------------------
    def slice(self, op_type, name, tensor_name, slice_specs, input_shape, output_shape):
        def bounds(spec, size):
            t = spec["type"]
            if t == "slice":
                s, e = spec.get("start"), spec.get("end")
                s = 0 if s is None else s
                e = size if e is None else e
            elif t == "index":
                s, e = spec["value"], spec["value"] + 1
            else:
                s, e = 0, size
            s = max(0, min(s, size))
            e = max(s, min(e, size))
            return s, e

        if len(input_shape) == 2 and len(slice_specs) <= 2:
            rows, cols = int(input_shape[0]), int(input_shape[1])
            rs_ = slice_specs[0] if len(slice_specs) > 0 else {"type": "full_slice"}
            cs_ = slice_specs[1] if len(slice_specs) > 1 else {"type": "full_slice"}
            r0, r1 = bounds(rs_, rows)
            c0, c1 = bounds(cs_, cols)
            return "", (f"{op_type}_2d", name, tensor_name, None, rows, cols, r0, r1, c0, c1,
                        max(0, r1 - r0), max(0, c1 - c0))
        if len(input_shape) == 1 and len(slice_specs) == 1:
            s, e = bounds(slice_specs[0], int(input_shape[0]))
            return "", (f"{op_type}_1d", name, tensor_name, None, s, max(0, e - s))
        raise NotImplementedError(f"slice of shape {tuple(input_shape)} with {len(slice_specs)} specs")

    def transpose(self, op_type, name, input_shape, tensor_name):
        if len(input_shape) == 2:
            return "", (f"{op_type}_2d", name, tensor_name, None, int(input_shape[0]),
                        int(input_shape[1]))
        raise NotImplementedError(f"transpose of shape {tuple(input_shape)}")

    def reshape(self, op_type, name, tensor_name, total_elements):
        return "", (f"{op_type}", name, tensor_name, None, total_elements)

    def concat(self, op_type, name, tensor_names, axis, env):
        if len(tensor_names) == 2 and axis == 0:
            t1, t2 = tensor_names
            s1, s2 = env[t1]["shape"], env[t2]["shape"]
            if len(s1) == 2:
                return "", (f"{op_type}_axis0", name, t1, t2, int(s1[0]), int(s2[0]), int(s1[1]))
        raise NotImplementedError(f"concat of {len(tensor_names)} tensors along axis {axis}")
