"""Device-buffer helpers for the GPU tests (torch is only the allocator).

Buffers made here stay referenced until finish(): a tensor created inline in
an argument list would otherwise be freed (and its block handed to the next
allocation) before the asynchronous kernel reads it."""
import numpy as np

_live = []


def dev(torch, array):
    """numpy -> CUDA tensor (same dtype), contiguous, kept alive until finish()."""
    a = np.ascontiguousarray(array)
    t = torch.from_numpy(a.copy()).cuda()
    _live.append(t)
    return t


def empty(torch, shape, dtype=np.float32):
    tdt = {np.float32: torch.float32, np.uint32: torch.int32, np.uint8: torch.uint8,
           np.int32: torch.int32}[np.dtype(dtype).type]
    t = torch.zeros(shape, dtype=tdt, device="cuda")
    _live.append(t)
    return t


def host(t, dtype=None):
    a = t.detach().cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a


def ptr(t):
    return t.data_ptr()


def call(lib, name, *args):
    import dav2_b200

    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise dav2_b200.Dav2CudaError(f"{name} -> {rc}: {lib.dav2cuda_last_error().decode()}")


def finish(torch, lib):
    torch.cuda.synchronize()
    err = lib.dav2cuda_device_error()
    _live.clear()
    assert err == 0, f"device error word = {err}"
