"""Guard bands around output tensors: a stand-in for the memory checkers
that are closed on the GPU pool.

``guarded(shape, dtype)`` returns an output tensor that is a slice of a
larger buffer whose bands before and after it hold a canary bit pattern (a
NaN with a payload no kernel produces); ``check()`` asserts that the bands
are still intact after the kernels ran, i.e. that nothing was written outside
the output -- partial-vector stores, out-of-range TMA rows, halo writes and
look-back tiles included.  Bands are 16-byte multiples, so the output keeps
the 16-byte alignment the library requires.
"""
import torch

_CANARY = {torch.float32: (torch.int32, 0x7FC0DEAD),
           torch.float16: (torch.int16, 0x7E5A),
           torch.bfloat16: (torch.int16, 0x7FDA)}


class Guarded:
    def __init__(self, shape, dtype, device="cuda", band_bytes=4096, fill=float("nan")):
        self.dtype = dtype
        n = 1
        for s in shape:
            n *= s
        es = torch.empty((), dtype=dtype).element_size()
        self.band = band_bytes // es
        ity, pattern = _CANARY[dtype]
        self.buf = torch.empty(n + 2 * self.band, dtype=dtype, device=device)
        self.buf.view(ity).fill_(pattern)
        self.pattern = pattern
        self.ity = ity
        self.out = self.buf[self.band:self.band + n].view(*shape)
        self.out.fill_(fill)

    def check(self, what=""):
        torch.cuda.synchronize()
        raw = self.buf.view(self.ity)
        n = self.out.numel()
        lo = raw[:self.band]
        hi = raw[self.band + n:]
        bad_lo = int((lo != self.pattern).sum())
        bad_hi = int((hi != self.pattern).sum())
        assert bad_lo == 0 and bad_hi == 0, (
            f"{what}: {bad_lo} element(s) written before and {bad_hi} after the output")


def guarded(shape, dtype, device="cuda", **kw):
    return Guarded(shape, dtype, device, **kw)
