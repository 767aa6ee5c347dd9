"""NumPy stand-in for ``mlx.core`` (golden-vector generation only).

Implements just the array surface that ``quantize_tensor`` /
``dequantize_tensor`` touch.  Semantics follow MLX's documented behaviour:
python scalars take the array's dtype; bf16/fp16 element-wise arithmetic is
computed in float32 and rounded (nearest-even) back to the dtype; ``round`` is
round-half-to-even; integer shifts wrap in the integer dtype.
"""

import numpy as np


def _round_bf16(a):
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32).reshape(a.shape)


class Dtype:
    def __init__(self, name, np_dtype, is_float, rank):
        self.name = name
        self.np = np_dtype
        self.is_float = is_float
        self.rank = rank

    def __repr__(self):
        return f"mlx.core.{self.name}"


uint8 = Dtype("uint8", np.uint8, False, 1)
int32 = Dtype("int32", np.int32, False, 3)
uint32 = Dtype("uint32", np.uint32, False, 3)
float16 = Dtype("float16", np.float32, True, 10)
bfloat16 = Dtype("bfloat16", np.float32, True, 10)
float32 = Dtype("float32", np.float32, True, 20)
bool_ = Dtype("bool", np.bool_, False, 0)


def _fit(values, dtype):
    """Bring float32 results into ``dtype``'s value set."""
    if dtype is bfloat16:
        return _round_bf16(values)
    if dtype is float16:
        return np.asarray(values, np.float32).astype(np.float16).astype(np.float32)
    if dtype.is_float:
        return np.asarray(values, np.float32)
    return np.asarray(values).astype(dtype.np)


def _promote(a, b):
    if a is b:
        return a
    if a.is_float and b.is_float:
        return float32
    if a.is_float:
        return a
    if b.is_float:
        return b
    return a if a.rank >= b.rank else b


class array:
    def __init__(self, data, dtype=None):
        if isinstance(data, array):
            dtype = dtype or data.dtype
            data = data._a
        a = np.asarray(data)
        if dtype is None:
            if a.dtype == np.bool_:
                dtype = bool_
            elif np.issubdtype(a.dtype, np.floating):
                dtype = float32
            elif a.dtype == np.uint8:
                dtype = uint8
            elif a.dtype == np.uint32:
                dtype = uint32
            else:
                dtype = int32
        self.dtype = dtype
        self._a = a if dtype is bool_ else _fit(a.astype(np.float32) if dtype.is_float else a, dtype)

    # -- basic attributes
    @property
    def shape(self):
        return tuple(self._a.shape)

    @property
    def size(self):
        return int(self._a.size)

    @property
    def ndim(self):
        return self._a.ndim

    def item(self):
        return self._a.item()

    def __array__(self, dtype=None, copy=None):
        return np.asarray(self._a, dtype=dtype)

    def astype(self, dtype):
        if dtype.is_float:
            return array(self._a.astype(np.float32), dtype)
        return array(self._a.astype(dtype.np), dtype)

    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return array(self._a.reshape(shape), self.dtype)

    def squeeze(self, axis=None):
        return array(np.squeeze(self._a, axis=axis), self.dtype)

    def __getitem__(self, idx):
        if isinstance(idx, array):
            idx = idx._a
        return array(self._a[idx], self.dtype)

    # -- arithmetic
    def _bin(self, other, fn, out_dtype=None):
        if isinstance(other, array):
            dt = _promote(self.dtype, other.dtype)
            ob = other._a
        else:
            dt = self.dtype if (self.dtype.is_float or isinstance(other, int)) else float32
            ob = other
        if dt.is_float:
            r = fn(self._a.astype(np.float32), np.asarray(ob, dtype=np.float32))
            return array(_fit(r, dt), dt) if out_dtype is None else array(r, out_dtype)
        r = fn(self._a.astype(dt.np), np.asarray(ob).astype(dt.np) if isinstance(other, array) else ob)
        return array(r, dt if out_dtype is None else out_dtype)

    def __add__(self, o):
        return self._bin(o, np.add)

    def __radd__(self, o):
        return self._bin(o, lambda a, b: np.add(b, a))

    def __sub__(self, o):
        return self._bin(o, np.subtract)

    def __rsub__(self, o):
        return self._bin(o, lambda a, b: np.subtract(b, a))

    def __mul__(self, o):
        return self._bin(o, np.multiply)

    def __rmul__(self, o):
        return self._bin(o, lambda a, b: np.multiply(b, a))

    def __truediv__(self, o):
        with np.errstate(divide="ignore", invalid="ignore"):
            return self._bin(o, np.divide)

    def __pow__(self, o):
        return self._bin(o, np.power)

    def __neg__(self):
        return array(-self._a, self.dtype)

    def __lshift__(self, o):
        return self._bin(o, np.left_shift)

    def __rshift__(self, o):
        return self._bin(o, np.right_shift)

    def __and__(self, o):
        return self._bin(o, np.bitwise_and)

    def __or__(self, o):
        return self._bin(o, np.bitwise_or)

    def __eq__(self, o):
        return self._bin(o, np.equal, out_dtype=bool_)

    def __gt__(self, o):
        return self._bin(o, np.greater, out_dtype=bool_)

    def __lt__(self, o):
        return self._bin(o, np.less, out_dtype=bool_)


def zeros(shape, dtype=float32):
    return array(np.zeros(shape, dtype=np.float32 if dtype.is_float else dtype.np), dtype)


def zeros_like(a):
    return zeros(a.shape, a.dtype)


def ones_like(a):
    return array(np.ones(a.shape, dtype=np.float32 if a.dtype.is_float else a.dtype.np), a.dtype)


def concatenate(arrs, axis=0):
    dt = arrs[0].dtype
    for a in arrs[1:]:
        dt = _promote(dt, a.dtype)
    return array(np.concatenate([a._a for a in arrs], axis=axis), dt)


def stack(arrs, axis=0):
    return array(np.stack([a._a for a in arrs], axis=axis), arrs[0].dtype)


def abs(a):  # noqa: A001 - mirrors the MLX name
    return array(np.abs(a._a), a.dtype)


def max(a, axis=None, keepdims=False):  # noqa: A001
    return array(np.max(a._a, axis=axis, keepdims=keepdims), a.dtype)


def mean(a, axis=None, keepdims=False):
    return array(np.mean(a._a.astype(np.float64), axis=axis, keepdims=keepdims).astype(np.float32), float32)


def where(cond, a, b):
    c = cond._a if isinstance(cond, array) else np.asarray(cond)
    dt = a.dtype if isinstance(a, array) else b.dtype
    av = a._a if isinstance(a, array) else a
    bv = b._a if isinstance(b, array) else b
    return array(np.where(c, av, bv), dt)


def round(a, decimals=0):  # noqa: A001
    return array(_fit(np.rint(a._a), a.dtype), a.dtype)


def clip(a, a_min, a_max):
    return array(_fit(np.clip(a._a, a_min, a_max), a.dtype), a.dtype)


# -- additions used by kv_compression.py / streaming_llm.py ---------------------
def _arr_tolist(self):
    return self._a.tolist()


array.tolist = _arr_tolist


def ones(shape, dtype=float32):
    return array(np.ones(shape, dtype=np.float32 if dtype.is_float else dtype.np), dtype)


def arange(start, stop=None, step=1, dtype=None):
    if stop is None:
        start, stop = 0, start
    return array(np.arange(start, stop, step).astype(np.int32), dtype or int32)


def argsort(a, axis=-1):
    # stable order for equal keys (lower position first)
    return array(np.argsort(a._a, axis=axis, kind="stable").astype(np.int32), int32)


def sort(a, axis=-1):
    return array(np.sort(a._a, axis=axis, kind="stable"), a.dtype)


def _getitem_ext(self, idx):
    if isinstance(idx, array):
        idx = idx._a
    elif isinstance(idx, tuple):
        idx = tuple(i._a if isinstance(i, array) else i for i in idx)
    return array(self._a[idx], self.dtype)


array.__getitem__ = _getitem_ext


def eval(*args):  # noqa: A001 - MLX's lazy-evaluation barrier; NumPy is eager
    return None
