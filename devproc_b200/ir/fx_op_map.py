"""FX target name → converter handler (reference: src/devproc/ir/fx_op_map.py:10-112).

Keys are the ``__name__`` of call_function targets (``.default`` stripped)
and call_method names; values name an ``FXToIRConverter._op_<value>``
handler.
"""

from typing import Dict


def get_fx_op_map() -> Dict[str, str]:
    m = {
        # contractions
        "linear": "linear", "matmul": "matmul", "mm": "matmul", "bmm": "matmul", "__matmul__": "matmul",
        "embedding": "embedding", "conv2d": "conv2d",
        "scaled_dot_product_attention": "sdpa",
        # activations
        "relu": "relu", "relu_": "relu", "sigmoid": "sigmoid", "tanh": "tanh", "gelu": "gelu",
        "silu": "silu", "exp": "exp", "neg": "neg",
        # arithmetic (torch functions, operator module and tensor methods)
        "add": "add", "iadd": "add", "__add__": "add", "__radd__": "add",
        "sub": "sub", "isub": "sub", "__sub__": "sub",
        "mul": "mul", "imul": "mul", "__mul__": "mul", "__rmul__": "mul",
        "truediv": "div", "div": "div", "__truediv__": "div",
        # reductions
        "softmax": "softmax", "argmax": "argmax", "mean": "mean", "sum": "sum", "amax": "amax",
        "layer_norm": "layer_norm", "rms_norm": "rms_norm",
        # casts and layout
        "to": "to", "float": "to", "half": "to", "bfloat16": "to", "int": "to", "long": "to", "type": "to",
        "contiguous": "passthrough", "clone": "passthrough", "detach": "passthrough",
        "view": "reshape", "reshape": "reshape", "flatten": "reshape", "unsqueeze": "reshape",
        "squeeze": "reshape", "permute": "permute", "transpose": "transpose", "t": "transpose",
        "interpolate": "interpolate",
        # slicing and joining
        "narrow": "narrow", "chunk": "chunk", "split": "split", "cat": "cat", "concat": "cat",
        "concatenate": "cat", "expand": "expand", "rope": "rope",
    }
    return m
