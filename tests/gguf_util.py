"""Test helper: write a GGUF file from a parameter dict {name: (ggml type,
shape, raw bytes)} with gguf-py 0.19.0, as the reference's converter does
(utils/convert-model/src/convert_hf_safetensors_to_gguf.py: GGUFWriter,
add_tensor with raw_dtype for BF16 / quantised bytes)."""
import gguf
import numpy as np
from gguf import GGMLQuantizationType as Q

GGML_F32, GGML_F16 = 0, 1


def _raw(data) -> bytes:
    if hasattr(data, "numpy"):  # synth parameters are CPU torch uint8 tensors
        return data.contiguous().numpy().tobytes()
    return bytes(data)


def _tensor_array(gtype, shape, data):
    raw = np.frombuffer(_raw(data), dtype=np.uint8)
    if gtype == GGML_F32:
        return raw.view(np.float32).reshape(shape), None
    if gtype == GGML_F16:
        return raw.view(np.float16).reshape(shape), None
    rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
    return raw.reshape(tuple(shape[:-1]) + (raw.size // rows,)), Q(gtype)


def write_gguf(path, params, alignment=None, kv=None, arch="flux2"):
    w = gguf.GGUFWriter(str(path), arch=arch)
    if alignment:
        w.add_custom_alignment(alignment)
    for k, (kind, v) in (kv or {}).items():
        getattr(w, "add_" + kind)(k, v)
    for name, (gtype, shape, data) in params.items():
        arr, raw_dtype = _tensor_array(gtype, shape, data)
        w.add_tensor(name, arr, raw_dtype=raw_dtype)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return str(path)
