"""A numpy stand-in for the handful of jax names flicker's hot path uses.

jax/jaxlib are not installed in this image and cannot be installed, so the
reference (pure JAX + Pallas) cannot run as shipped. To still execute the
reference's OWN source for ``kernels.qk_prep``, ``kernels.attend``,
``modules.qkv_prep``, ``nn.sdpa``, ``rope.*`` and ``loader.check_logit_bound``
when generating golden vectors, ``install()`` registers tiny modules named
``jax``, ``jax.numpy``, ``jax.lax``, ``jax.nn`` and ``jax.experimental.pallas``
(+ ``.tpu``) that map those names onto numpy / ml_dtypes:

* ``jnp.*`` -> numpy (fp32 arithmetic, bf16 via ``ml_dtypes`` with
  round-to-nearest-even, as ``astype(jnp.bfloat16)`` does);
* ``lax.rsqrt``/``dot``/``dot_general``/``broadcasted_iota`` -> numpy with fp32
  accumulation (``preferred_element_type=float32``);
* ``pl.pallas_call`` -> a sequential grid interpreter: it walks the grid in
  row-major order (last axis fastest, as Pallas does on one core), hands the
  kernel body numpy VIEWS of each block chosen by the BlockSpec index maps,
  and keeps scratch buffers alive across grid steps.

Used only by ``make_golden.py`` in this folder, never by the package or the
GPU tests. What this pins: the reference's algorithm, operation order,
tiling and rounding points. What it cannot pin: XLA's own transcendental
ulps (``exp``, ``cos``, ``rsqrt``), which numpy supplies here.
"""
from __future__ import annotations

import sys
import types

import ml_dtypes
import numpy as np

_STATE = {"program_id": ()}


class ShapeDtypeStruct:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)


class BlockSpec:
    def __init__(self, block_shape, index_map):
        self.block_shape = tuple(block_shape)
        self.index_map = index_map


class PrefetchScalarGridSpec:
    def __init__(self, num_scalar_prefetch, grid, in_specs, out_specs, scratch_shapes=()):
        assert num_scalar_prefetch == 0
        self.grid = tuple(grid)
        self.in_specs = in_specs
        self.out_specs = out_specs
        self.scratch_shapes = list(scratch_shapes)


class _Vmem:
    def __init__(self, shape, dtype):
        self.shape = tuple(shape)
        self.dtype = np.dtype(dtype)


def _block(arr: np.ndarray, spec: BlockSpec, idx) -> np.ndarray:
    blocks = spec.index_map(*idx)
    sl = tuple(slice(b * s, (b + 1) * s) for b, s in zip(blocks, spec.block_shape))
    view = arr[sl]
    assert view.shape == spec.block_shape, (view.shape, spec.block_shape)
    return view


def pallas_call(kernel, out_shape, grid=None, in_specs=None, out_specs=None, grid_spec=None,
                compiler_params=None, interpret=False, name=None):
    single = not isinstance(out_shape, (list, tuple))
    shapes = [out_shape] if single else list(out_shape)
    scratch_shapes = []
    if grid_spec is not None:
        grid, in_specs, out_specs = grid_spec.grid, grid_spec.in_specs, grid_spec.out_specs
        scratch_shapes = grid_spec.scratch_shapes
    out_list = [out_specs] if single else list(out_specs)

    def run(*args):
        outs = [np.zeros(s.shape, s.dtype) for s in shapes]
        scratch = [np.zeros(s.shape, s.dtype) for s in scratch_shapes]
        for idx in np.ndindex(*grid):
            _STATE["program_id"] = idx
            ins = [_block(np.asarray(a), sp, idx) for a, sp in zip(args, in_specs)]
            o = [_block(a, sp, idx) for a, sp in zip(outs, out_list)]
            kernel(*ins, *o, *scratch)
        return outs[0] if single else outs

    return run


def _program_id(axis: int) -> int:
    return _STATE["program_id"][axis]


def _when(cond):
    def deco(fn):
        if bool(cond):
            fn()
        return fn
    return deco


def _softmax(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def _dot_general(a, b, dims, preferred_element_type=None):
    (ca, cb), (ba, bb) = dims
    assert not ba and not bb
    t = preferred_element_type or np.result_type(a.dtype, b.dtype)
    return np.tensordot(np.asarray(a, t), np.asarray(b, t), axes=(list(ca), list(cb))).astype(t)


def _dot(a, b, preferred_element_type=None):
    t = preferred_element_type or np.result_type(a.dtype, b.dtype)
    return (np.asarray(a, t) @ np.asarray(b, t)).astype(t)


def _iota(dtype, shape, dimension):
    ar = np.arange(shape[dimension], dtype=dtype)
    view = [1] * len(shape)
    view[dimension] = shape[dimension]
    return np.broadcast_to(ar.reshape(view), shape)


def _rsqrt(x):
    x = np.asarray(x)
    return (np.asarray(1.0, x.dtype) / np.sqrt(x)).astype(x.dtype)


def install() -> None:
    """Register the stand-in modules in ``sys.modules`` (idempotent)."""
    if getattr(sys.modules.get("jax"), "_flicker_stand_in", False):
        return
    jax = types.ModuleType("jax")
    jax._flicker_stand_in = True
    jnp = types.ModuleType("jax.numpy")
    for name in ("arange", "stack", "cos", "sin", "concatenate", "repeat", "mean", "where", "exp",
                 "sum", "zeros", "max", "abs", "square", "einsum", "inf", "float32", "int32",
                 "split", "maximum", "full", "ones", "sqrt", "asarray"):
        setattr(jnp, name, getattr(np, name))
    jnp.bfloat16 = ml_dtypes.bfloat16
    jnp.float16 = np.float16
    jnp.uint8 = np.uint8
    lax = types.ModuleType("jax.lax")
    lax.rsqrt = _rsqrt
    lax.dot_general = _dot_general
    lax.dot = _dot
    lax.broadcasted_iota = _iota
    nn = types.ModuleType("jax.nn")
    nn.softmax = _softmax
    nn.silu = lambda x: x / (1.0 + np.exp(-x))
    nn.gelu = lambda x: x
    experimental = types.ModuleType("jax.experimental")
    pl = types.ModuleType("jax.experimental.pallas")
    pl.BlockSpec = BlockSpec
    pl.pallas_call = pallas_call
    pl.program_id = _program_id
    pl.when = _when
    pltpu = types.ModuleType("jax.experimental.pallas.tpu")
    pltpu.roll = lambda x, shift, axis: np.roll(x, shift, axis=axis)
    pltpu.PrefetchScalarGridSpec = PrefetchScalarGridSpec
    pltpu.VMEM = _Vmem
    pltpu.CompilerParams = lambda **kw: kw
    pl.tpu = pltpu
    experimental.pallas = pl
    jax.numpy, jax.lax, jax.nn, jax.experimental = jnp, lax, nn, experimental
    jax.Array = np.ndarray
    jax.ShapeDtypeStruct = ShapeDtypeStruct
    jax.device_put = lambda x, *a, **k: x
    jax.default_backend = lambda: "cpu"
    sys.modules.update({
        "jax": jax, "jax.numpy": jnp, "jax.lax": lax, "jax.nn": nn,
        "jax.experimental": experimental, "jax.experimental.pallas": pl,
        "jax.experimental.pallas.tpu": pltpu,
    })
