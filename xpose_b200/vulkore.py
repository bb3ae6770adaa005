"""Python mirror of the reference runtime surface the decode loop uses
(include/vulkore/{context,buffer,program,launch,sync}.hpp), over the C ABI.

    ctx  = Context()
    prog = Program.from_file(ctx, "kernels/llm_matvec.spv")
    mv   = prog.kernel("mv_km4_bs")               # unknown name -> XpError
    launch(mv, Grid(cols), out, x, wq, sc, rows, cols).wait()
    b = Batch(ctx); b.add(...); b.add(...); b.submit().wait()

Arguments are matched positionally against the kernel's signature exactly as
vulkore::launch does (src/launch.cpp:63-131): a Buffer (or a CUDA torch
tensor) for a global pointer, a POD for a push constant, with the POD's byte
size checked (Python int -> uint32, float -> fp32; numpy scalars keep their
own size, so np.float64(2.0) for a float argument is the reference's
"double literal for a float arg" error).
"""
import ctypes as C

import numpy as np

from ._lib import XP_OK, XP_TIMEOUT, Arg, Grid as _CGrid, XpError, check, lib

Error = XpError


class Usage:
    DeviceLocal = 0
    HostVisible = 1


def Grid(x, y=1, z=1):
    """Global thread counts (CUDA semantics), as vulkore::Grid."""
    return _CGrid(x, y, z)


class Context:
    def __init__(self, device=0):
        h = C.c_void_p()
        check(lib().xp_context_create(device, C.byref(h)))
        self._h = h
        self.device = device

    @property
    def handle(self):
        return self._h

    @property
    def stream(self):
        return lib().xp_context_stream(self._h)

    def device_name(self):
        buf = C.create_string_buffer(256)
        check(lib().xp_context_device_name(self._h, buf, 256))
        return buf.value.decode()

    def alloc(self, count, dtype=np.float32, usage=Usage.DeviceLocal):
        dtype = np.dtype(dtype)
        if dtype.itemsize % 4:
            raise XpError(-1, "storage buffer element types should be 4-byte aligned")
        return Buffer(self, int(count) * dtype.itemsize, usage, dtype)

    def wait_idle(self):
        check(lib().xp_context_wait_idle(self._h))

    def close(self):
        if self._h:
            lib().xp_context_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Buffer:
    def __init__(self, ctx, nbytes, usage, dtype):
        d, h = C.c_void_p(), C.c_void_p()
        check(lib().xp_alloc(ctx.handle, nbytes, usage, C.byref(d), C.byref(h)))
        self.ctx, self.ptr, self.host, self.nbytes, self.dtype, self.usage = ctx, d.value, h.value, nbytes, dtype, usage

    def size_bytes(self):
        return self.nbytes

    def host_visible(self):
        return self.usage == Usage.HostVisible

    def upload(self, arr, offset_bytes=0):
        a = np.ascontiguousarray(arr)
        if offset_bytes + a.nbytes > self.nbytes:
            raise XpError(-1, "Buffer::upload out of range")
        check(lib().xp_upload(self.ctx.handle, self.ptr, offset_bytes, a.ctypes.data, a.nbytes))

    def download(self, count=None, dtype=None, offset_bytes=0):
        dtype = np.dtype(dtype or self.dtype)
        count = count if count is not None else (self.nbytes - offset_bytes) // dtype.itemsize
        out = np.empty(count, dtype)
        if offset_bytes + out.nbytes > self.nbytes:
            raise XpError(-1, "Buffer::download out of range")
        check(lib().xp_download(self.ctx.handle, out.ctypes.data, self.ptr, offset_bytes, out.nbytes))
        return out

    def free(self):
        if self.ptr:
            lib().xp_free(self.ctx.handle, self.ptr)
            self.ptr = None


class Kernel:
    def __init__(self, kid):
        self.id = kid
        mod, name, n = C.c_char_p(), C.c_char_p(), C.c_uint32()
        check(lib().xp_kernel_info(kid, C.byref(mod), C.byref(name), C.byref(n)))
        self.module, self.name, self.nargs = mod.value.decode(), name.value.decode(), n.value

    def valid(self):
        return self.id >= 0

    def args(self):
        out = []
        for i in range(self.nargs):
            kind, size, nm = C.c_int(), C.c_uint32(), C.c_char_p()
            check(lib().xp_kernel_arg(self.id, i, C.byref(kind), C.byref(size), C.byref(nm)))
            out.append((kind.value, size.value, nm.value.decode()))
        return out


class Program:
    """A module path -> kernel-by-name registry (include/vulkore/program.hpp)."""

    def __init__(self, ctx, module):
        self.ctx, self.module = ctx, module

    @staticmethod
    def from_file(ctx, path):
        return Program(ctx, path)

    def kernel(self, name):
        kid = C.c_int32()
        check(lib().xp_kernel_lookup(self.module.encode(), name.encode(), C.byref(kid)))
        return Kernel(kid.value)

    def kernel_names(self):
        names = []
        for i in range(lib().xp_kernel_count()):
            k = Kernel(i)
            if k.module.split("/")[-1] == self.module.split("/")[-1]:
                names.append(k.name)
        return names


def _marshal(args):
    keep = []
    arr = (Arg * max(1, len(args)))()
    for i, a in enumerate(args):
        if isinstance(a, Buffer):
            arr[i] = Arg(a.ptr, 0, 1)
        elif hasattr(a, "data_ptr") and hasattr(a, "is_cuda"):
            arr[i] = Arg(a.data_ptr(), 0, 1)
        else:
            if isinstance(a, np.generic):
                v = np.array(a)
                keep.append(v)
                arr[i] = Arg(v.ctypes.data, v.nbytes, 0)
                continue
            if isinstance(a, bool):
                v = C.c_uint32(int(a))
            elif isinstance(a, int):
                v = C.c_uint32(a)
            elif isinstance(a, float):
                v = C.c_float(a)
            else:
                raise TypeError(f"argument {i}: pass a Buffer, a CUDA tensor or a POD value, got {type(a)}")
            keep.append(v)
            arr[i] = Arg(C.addressof(v), C.sizeof(v), 0)
    return arr, keep


class Fence:
    def __init__(self, h):
        self._h = h

    def wait(self, timeout_ns=2**64 - 1):
        """True when signaled, False on timeout; raises on a device error."""
        s = lib().xp_fence_wait(self._h, C.c_uint64(timeout_ns))
        if s == XP_TIMEOUT:
            return False
        check(s)
        return True

    def __del__(self):
        try:
            if self._h:
                lib().xp_fence_destroy(self._h)  # the destructor drains
                self._h = None
        except Exception:
            pass


class _DoneFence:
    def wait(self, timeout_ns=2**64 - 1):
        return True


def launch(kernel, grid, *args, stream=None):
    """vulkore::launch: validate, enqueue, return a Fence."""
    arr, keep = _marshal(args)
    check(lib().xp_launch(kernel.id, grid, arr, len(args), stream))
    return _DoneFence()


class Batch:
    """Many launches, one CUDA graph launch (vulkore::Batch)."""

    def __init__(self, ctx):
        h = C.c_void_p()
        check(lib().xp_batch_create(ctx.handle, C.byref(h)))
        self._h = h

    def add(self, kernel, grid, *args):
        arr, keep = _marshal(args)
        check(lib().xp_batch_add(self._h, kernel.id, grid, arr, len(args)))
        return self

    def size(self):
        n = C.c_uint32()
        check(lib().xp_batch_size(self._h, C.byref(n)))
        return n.value

    def submit(self):
        f = C.c_void_p()
        check(lib().xp_batch_submit(self._h, C.byref(f)))
        return Fence(f)

    def __del__(self):
        try:
            if self._h:
                lib().xp_batch_destroy(self._h)
                self._h = None
        except Exception:
            pass
