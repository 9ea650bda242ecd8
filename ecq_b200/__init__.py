"""ecq_b200 -- B200 (sm_100a) implementation of ecq's hot path: interleaved
rANS decode of 4-bit weight symbols fused with per-group dequantisation and
the GEMV that consumes them, behind the reference's Python interface.

Host-side codec:   RANSTable, InterleavedEncodedTile, interleaved_rans_encode,
                   InterleavedRANSEncoder, encode_matrix
GPU decode:        interleaved_rans_decode, InterleavedRANSDecoder,
                   CudaInterleavedRANS, DeviceMatrix.decode
Fused GEMV:        DeviceMatrix.gemv, entropy_coded_matmul, EntropyCodedLinear
Plain 4-bit:       Packed4Matrix (the CACHED store and the HBM-bound control)
"""
from .codec import (EncodedMatrix, InterleavedEncodedTile, InterleavedRANSEncoder, RANSTable,  # noqa: F401
                    encode_matrix, interleaved_rans_encode, pack_reference_tiles, choose_tile_cols)

PROB_BITS = 14
PROB_SCALE = 1 << PROB_BITS
RANS_BYTE_L = 1 << 23


def __getattr__(name):
    # GPU-side modules import torch; load them on first use
    if name in ("DeviceMatrix", "Packed4Matrix", "device_info"):
        from . import device
        return getattr(device, name)
    if name in ("interleaved_rans_decode", "InterleavedRANSDecoder", "CudaInterleavedRANS",
                "verify_interleaved_roundtrip"):
        from . import interleaved
        return getattr(interleaved, name)
    if name in ("entropy_coded_matmul", "EntropyCodedLinear", "rans_gemv", "rans_matmul"):
        from . import ops
        return getattr(ops, name)
    if name in ("SmartDecoder", "DecodeMode", "DecodedWeights"):
        from . import strategies
        return getattr(strategies, name)
    raise AttributeError(name)
