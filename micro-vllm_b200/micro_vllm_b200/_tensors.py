"""Small tensor helpers shared by the host wrappers (no compute)."""
import torch

from . import _native

DTYPE_CODES = {
    torch.float32: _native.DTYPE_F32,
    torch.float16: _native.DTYPE_F16,
    torch.bfloat16: _native.DTYPE_BF16,
}

INDEX_CODES = {
    torch.int32: _native.INDEX_I32,
    torch.int64: _native.INDEX_I64,
}


def storage_overlaps(left: torch.Tensor, right: torch.Tensor) -> bool:
    """True when the two tensors' storages share any byte.

    Compares byte intervals of the underlying storages rather than storage
    identity, so aliases created through DLPack (independent storage objects
    over the same memory) are caught too.
    """
    left_storage, right_storage = left.untyped_storage(), right.untyped_storage()
    left_size, right_size = left_storage.nbytes(), right_storage.nbytes()
    if left_size == 0 or right_size == 0:
        return False
    left_start, right_start = left_storage.data_ptr(), right_storage.data_ptr()
    if left_start <= right_start:
        return right_start - left_start < left_size
    return left_start - right_start < right_size


def current_stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# The raw handle of the current stream of a device index, without building a
# torch.cuda.Stream object (torch's own fast accessor where this build has it).
_raw_stream = getattr(torch._C, '_cuda_getCurrentRawStream', None)


def current_stream_raw(device_index: int) -> int:
    if _raw_stream is not None:
        return _raw_stream(device_index)
    return torch.cuda.current_stream(device_index).cuda_stream
