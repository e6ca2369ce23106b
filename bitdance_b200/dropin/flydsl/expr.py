"""Element-type tags the reference's scripts pass to from_c_void_p (kernel/verify_w4a6.py:28-31,
kernel/bench_sweep.py:21-24). They only label pointers here."""


class DType:
    __slots__ = ("name", "bits")

    def __init__(self, name, bits):
        self.name = name
        self.bits = bits

    def __repr__(self):
        return self.name


Int8 = DType("Int8", 8)
Int16 = DType("Int16", 16)
Int32 = DType("Int32", 32)
Float32 = DType("Float32", 32)
BFloat16 = DType("BFloat16", 16)
