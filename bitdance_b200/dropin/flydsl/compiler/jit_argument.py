"""``from_c_void_p(dtype, ptr)``: the reference wraps a device pointer with its element type
(kernel/verify_w4a6.py:35-36). The launcher reads the address from ``.value``."""


class CVoidPtr:
    __slots__ = ("dtype", "value")

    def __init__(self, dtype, ptr):
        self.dtype = dtype
        self.value = int(ptr)

    def __repr__(self):
        return f"CVoidPtr({self.dtype!r}, 0x{self.value:x})"


def from_c_void_p(dtype, ptr) -> CVoidPtr:
    return CVoidPtr(dtype, ptr)
