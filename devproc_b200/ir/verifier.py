"""IR verifier: SSA, def-use, per-op type rules and devices.

Same checks and messages as the reference (src/devproc/ir/verifier.py:38-389)
for the ops both know, extended to the ops this build adds.  ``verify()``
returns a bool and collects the messages in ``get_errors()``.
"""

from typing import List, Set

from .function import Function
from .types import DictType, ScalarType, StringType, TensorType, TokenizerType


class IRVerifier:
    def __init__(self, function: Function):
        self.function = function
        self.errors: List[str] = []

    def verify(self) -> bool:
        self.errors = []
        self._check_ssa()
        self._check_def_use()
        self._check_types()
        self._check_devices()
        return not self.errors

    def get_errors(self) -> List[str]:
        return self.errors

    # ------------------------------------------------------------------
    def _check_ssa(self) -> None:
        seen: Set[str] = set()
        for v in self.function.inputs:
            if v.name in seen:
                self.errors.append(f"SSA violation: input '{v.name}' defined multiple times")
            seen.add(v.name)
        for op in self.function.block.ops:
            for v in op.outputs:
                if v.name in seen:
                    self.errors.append(
                        f"SSA violation: value '{v.name}' defined multiple times (at op: {op.name})")
                seen.add(v.name)

    def _check_def_use(self) -> None:
        defined: Set[str] = {v.name for v in self.function.inputs}
        for op in self.function.block.ops:
            for v in op.outputs:
                defined.add(v.name)
            for v in op.inputs:
                if v.name not in defined:
                    self.errors.append(
                        f"Def-use error: value '{v.name}' used in op '{op.name}' but never defined")

    def _need(self, cond: bool, msg: str) -> bool:
        if not cond:
            self.errors.append(msg)
        return cond

    def _check_types(self) -> None:
        for op in self.function.block.ops:
            check = getattr(self, "_t_" + op.name, None)
            if check is not None:
                check(op)

    # per-op rules -------------------------------------------------------
    def _t_normalize(self, op) -> None:
        if not self._need(len(op.outputs) == 1,
                          f"normalize should have exactly 1 output, got {len(op.outputs)}"):
            return
        t = op.outputs[0].type
        if not self._need(isinstance(t, TensorType),
                          f"normalize output must be TensorType, got {type(t)}"):
            return
        self._need(t.dtype == "float32", f"normalize output dtype must be float32, got {t.dtype}")

    def _t_argmax(self, op) -> None:
        if not self._need(len(op.outputs) == 1,
                          f"argmax should have exactly 1 output, got {len(op.outputs)}"):
            return
        t = op.outputs[0].type
        if isinstance(t, ScalarType):
            self._need(t.dtype == "int64", f"argmax output dtype must be int64, got {t.dtype}")
        elif isinstance(t, TensorType):
            self._need(t.dtype in ("int32", "int64"),
                       f"argmax output dtype must be int32 or int64, got {t.dtype}")
        else:
            self.errors.append(f"argmax output must be ScalarType, got {type(t)}")

    def _t_matmul(self, op) -> None:
        if not self._need(len(op.inputs) == 2, f"matmul requires 2 inputs, got {len(op.inputs)}"):
            return
        a, b = op.inputs[0].type, op.inputs[1].type
        if not self._need(isinstance(a, TensorType) and isinstance(b, TensorType),
                          "matmul requires TensorType inputs"):
            return
        if not self._need(len(a.shape) >= 2 and len(b.shape) >= 2, "matmul requires 2D tensors"):
            return
        self._need(a.shape[-1] == b.shape[-2],
                   f"matmul dimension mismatch: {a.shape[-1]} != {b.shape[-2]}")

    def _t_linear(self, op) -> None:
        if not self._need(len(op.inputs) in (2, 3), "linear requires 2 or 3 inputs"):
            return
        x, w = op.inputs[0].type, op.inputs[1].type
        if self._need(isinstance(x, TensorType) and isinstance(w, TensorType),
                      "linear requires TensorType inputs"):
            self._need(x.shape[-1] == w.shape[-1],
                       f"linear dimension mismatch: {x.shape[-1]} != {w.shape[-1]}")

    def _t_relu(self, op) -> None:
        if not self._need(len(op.inputs) == 1 and len(op.outputs) == 1,
                          "relu requires 1 input and 1 output"):
            return
        i, o = op.inputs[0].type, op.outputs[0].type
        if not self._need(isinstance(i, TensorType) and isinstance(o, TensorType),
                          "relu requires TensorType"):
            return
        self._need(i.shape == o.shape, f"relu: input shape {i.shape} != output shape {o.shape}")

    def _t_load_tokenizer(self, op) -> None:
        if self._need(len(op.outputs) == 1, "load_tokenizer should have 1 output"):
            self._need(isinstance(op.outputs[0].type, TokenizerType),
                       "load_tokenizer output must be TokenizerType")

    def _t_tokenize_encode(self, op) -> None:
        if not self._need(len(op.inputs) == 2, "tokenize_encode requires 2 inputs"):
            return
        if not self._need(len(op.outputs) == 1, "tokenize_encode requires 1 output"):
            return
        self._need(isinstance(op.inputs[0].type, TokenizerType),
                   "tokenize_encode input 0 must be TokenizerType")
        self._need(isinstance(op.inputs[1].type, StringType),
                   "tokenize_encode input 1 must be StringType")
        self._need(isinstance(op.outputs[0].type, TensorType),
                   "tokenize_encode output must be TensorType")

    def _t_tokenize_decode(self, op) -> None:
        if not self._need(len(op.inputs) == 2, "tokenize_decode requires 2 inputs"):
            return
        if not self._need(len(op.outputs) == 1, "tokenize_decode requires 1 output"):
            return
        self._need(isinstance(op.inputs[0].type, TokenizerType),
                   "tokenize_decode input 0 must be TokenizerType")
        self._need(isinstance(op.inputs[1].type, TensorType),
                   "tokenize_decode input 1 must be TensorType")
        self._need(isinstance(op.outputs[0].type, StringType),
                   "tokenize_decode output must be StringType")

    def _t_string_length(self, op) -> None:
        if not self._need(len(op.inputs) == 1, "string_length requires 1 input"):
            return
        if not self._need(len(op.outputs) == 1, "string_length requires 1 output"):
            return
        self._need(isinstance(op.inputs[0].type, StringType), "string_length input must be StringType")
        self._need(isinstance(op.outputs[0].type, ScalarType), "string_length output must be ScalarType")

    def _t_string_concat(self, op) -> None:
        if not self._need(len(op.inputs) == 2, "string_concat requires 2 inputs"):
            return
        if not self._need(len(op.outputs) == 1, "string_concat requires 1 output"):
            return
        self._need(isinstance(op.inputs[0].type, StringType), "string_concat input 0 must be StringType")
        self._need(isinstance(op.inputs[1].type, StringType), "string_concat input 1 must be StringType")
        self._need(isinstance(op.outputs[0].type, StringType), "string_concat output must be StringType")

    def _t_string_slice(self, op) -> None:
        if not self._need(len(op.inputs) == 1, "string_slice requires 1 input"):
            return
        if not self._need(len(op.outputs) == 1, "string_slice requires 1 output"):
            return
        self._need(isinstance(op.inputs[0].type, StringType), "string_slice input must be StringType")
        self._need(isinstance(op.outputs[0].type, StringType), "string_slice output must be StringType")

    def _t_string_format(self, op) -> None:
        if not self._need(len(op.inputs) >= 1, "string_format requires at least 1 input"):
            return
        if not self._need(len(op.outputs) == 1, "string_format requires 1 output"):
            return
        self._need(isinstance(op.inputs[0].type, StringType), "string_format input 0 must be StringType")
        self._need(isinstance(op.outputs[0].type, StringType), "string_format output must be StringType")

    def _t_dict_create(self, op) -> None:
        if self._need(len(op.outputs) == 1, "dict_create requires 1 output"):
            self._need(isinstance(op.outputs[0].type, DictType), "dict_create output must be DictType")

    def _t_dict_get(self, op) -> None:
        if not self._need(len(op.inputs) == 2, "dict_get requires 2 inputs"):
            return
        if self._need(len(op.outputs) == 1, "dict_get requires 1 output"):
            self._need(isinstance(op.inputs[0].type, DictType), "dict_get input 0 must be DictType")

    def _t_dict_set(self, op) -> None:
        if not self._need(len(op.inputs) == 3, "dict_set requires 3 inputs"):
            return
        if not self._need(len(op.outputs) == 1, "dict_set requires 1 output"):
            return
        self._need(isinstance(op.inputs[0].type, DictType), "dict_set input 0 must be DictType")
        self._need(isinstance(op.outputs[0].type, DictType), "dict_set output must be DictType")

    def _t_dict_size(self, op) -> None:
        if not self._need(len(op.inputs) == 1, "dict_size requires 1 input"):
            return
        if not self._need(len(op.outputs) == 1, "dict_size requires 1 output"):
            return
        self._need(isinstance(op.inputs[0].type, DictType), "dict_size input must be DictType")
        self._need(isinstance(op.outputs[0].type, ScalarType), "dict_size output must be ScalarType")

    # ------------------------------------------------------------------
    def _check_devices(self) -> None:
        valid = TensorType.VALID_DEVICES
        for v in self.function.inputs:
            if isinstance(v.type, TensorType) and v.type.device not in valid:
                self.errors.append(f"Invalid device '{v.type.device}' for value '{v.name}'")
        for op in self.function.block.ops:
            for v in op.outputs:
                if isinstance(v.type, TensorType) and v.type.device not in valid:
                    self.errors.append(f"Invalid device '{v.type.device}' for value '{v.name}'")
