"""GGUF checkpoints: reader, writer, block quantizers, random-init model synthesis."""
from .constants import BLOCK_INFO, GGMLType, QK_K, ValueType, tensor_nbytes
from .quants import dequantize, quantize
from .reader import GGUFError, GGUFFile, TensorInfo, open_gguf
from .writer import GGUFWriter

__all__ = [
    "BLOCK_INFO", "GGMLType", "QK_K", "ValueType", "tensor_nbytes", "dequantize", "quantize",
    "GGUFError", "GGUFFile", "TensorInfo", "open_gguf", "GGUFWriter",
]
