"""GPU parity for binary ops on operands of different dtypes, where the promotion is fused into the op
(mtxc_broadcast_binary_mixed: a Float result with one Float operand).  The reference evaluates
astype(promote_types(a, b)) of the other operand and then the op; the oracle does exactly that, and the
fused kernel must give the same bits."""
import numpy as np
import pytest

from tests.helpers import assert_bits_equal
from tests.test_gpu_pointwise import dev
from tests.test_oracle_pin_pointwise import values

pytestmark = pytest.mark.gpu

OTHER = [1, 2, 3, 4, 5, 6, 7, 8, 10, 11, 12]  # every dtype but Float and Complex64
LAYOUTS = [([64, 1, 1024], [1, 16, 1024]), ([5], [3, 5]), ([7, 13], [7, 13]), ([4, 4096], [4096]), ([], [6])]


@pytest.mark.parametrize("code", OTHER)
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div", "equal"])
def test_mixed_float_and_other(gpu, port, code, op):
    rng = np.random.default_rng(400 + code)
    for sf, so in LAYOUTS:
        f = values(rng, 0, int(np.prod(sf)), special=True).reshape(sf)
        o = values(rng, code, int(np.prod(so)), special=code in (1, 10)).reshape(so)
        if op == "equal":  # make some pairs equal after the conversion
            fo = port.astype(o, np.float32, src_code=code, dst_code=0)
            k = min(f.size, fo.size) // 2
            f.reshape(-1)[:k] = fo.reshape(-1)[:k]
        o_as_f = port.astype(o, np.float32, src_code=code, dst_code=0)
        for a, b, ad, bd, tag in ((f, o_as_f, dev(f, 0), dev(o, code), "float op other"),
                                  (o_as_f, f, dev(o, code), dev(f, 0), "other op float")):
            want = port.binary(op, np.ascontiguousarray(a), np.ascontiguousarray(b))
            got = gpu.binary(op, ad, bd)
            gpu.sync()
            assert str(got.dtype) == "torch.float32"
            assert_bits_equal(got.cpu().numpy(), want, f"{tag}: {op} code {code} {sf} {so}")


def test_mixed_strided_and_transposed(gpu, port):
    import torch

    rng = np.random.default_rng(77)
    f = values(rng, 0, 40 * 33, special=True).reshape(40, 33)
    i = values(rng, 3, 33 * 40).reshape(33, 40)
    fd, idv = dev(f, 0), dev(i, 3)
    got = gpu.binary("mul", fd, idv.T)  # a transposed int32 operand
    gpu.sync()
    want = port.binary("mul", f, port.astype(i.T, np.float32, make_contig=False, src_code=3, dst_code=0))
    assert_bits_equal(got.cpu().numpy(), want, "mul f32 x int32^T")
    with pytest.raises(Exception):
        gpu.binary("max", fd, idv.T)  # max / min do not promote
    assert torch.cuda.is_available()
