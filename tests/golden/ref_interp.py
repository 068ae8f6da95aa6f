"""Run the reference's own Triton-Ascend SFA kernels on the CPU (fixture generation only).

The reference (lilac-me/ops ``SFA.py``) targets Ascend NPUs through Triton-Ascend.
Its kernel bodies are plain ``triton.language`` plus three Ascend extensions, so
they execute under Triton's CPU interpreter once those extensions are emulated:

* ``al.sub_vec_id()`` — the Ascend cube core drives two vector sub-cores; each
  program body runs here in two Python threads with ids 0 and 1 that share the
  per-program global-memory workspaces, as the two sub-cores do.
* ``al.sync_block_set/wait`` — cube/vector hand-off flags; a two-party barrier.
* ``torch_npu`` and ``triton.extension.buffer.language`` — imported, unused.

Three interpreter gaps are patched (all value-preserving): ``tl.dot`` on bf16
operands (the interpreter multiplies raw 16-bit patterns), fp16<->bf16 casts
(routed through fp32), and the power-of-two block-shape rule (the reference uses
BLOCK_N = 80).  Loop counters become interpreter scalars because the kernels call
``.to(tl.float32)`` on them (``SFA.py:389``).

This module imports the reference source from a path given by the caller; it is
used only by ``make_golden.py`` in the container that holds the reference and is
never imported by tests, the bench or the product.
"""
from __future__ import annotations

import builtins
import inspect
import os
import sys
import threading
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import triton  # noqa: E402
import triton.language as tl  # noqa: E402


def _install_stubs():
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    for name in ("triton.extension", "triton.extension.buffer", "triton.extension.buffer.language",
                 "triton.language.extra.cann"):
        sys.modules.setdefault(name, types.ModuleType(name))
    al = types.ModuleType("triton.language.extra.cann.extension")
    state = threading.local()
    barrier = [None]

    from triton.runtime.interpreter import TensorHandle

    def scalar(i):
        return tl.core.tensor(TensorHandle(np.array([i], dtype=np.int32).reshape(()), tl.int32), tl.int32)

    al.sub_vec_id = lambda: scalar(state.sid)
    al.sync_block_set = lambda *a: None
    al.sync_block_wait = lambda *a: barrier[0].wait()
    sys.modules["triton.language.extra.cann.extension"] = al
    return state, barrier, scalar


def load_reference(ref_dir: str):
    """Import ``SFA.py`` from ``ref_dir`` with the emulation installed; returns the module."""
    state, barrier, scalar = _install_stubs()
    import triton.runtime.interpreter as I
    import triton.language.semantic as SEM
    import triton.language.core as CORE

    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import SFA  # the reference module, unchanged

    extra = set(SFA._COMMMON_EXTRA_ARGS)

    class TwoSubCoreExecutor(I.GridExecutor):
        def __call__(self, *args_dev, **kwargs):
            argspec = inspect.getfullargspec(self.fn)
            kwargs = {k: v for k, v in kwargs.items() if k in argspec.args}
            args_hst, kwargs_hst = self._init_args_hst(args_dev, kwargs)
            scope = I._patch_lang(self.fn)
            try:
                args = inspect.getcallargs(self.fn, *args_hst, **kwargs_hst)
                args = {n: a if n in self.constexprs else I._implicit_cvt(a) for n, a in args.items()}
                grid = tuple(self.grid) + (1,) * (3 - len(self.grid))
                I.interpreter_builder.set_grid_dim(*grid)
                for x in builtins.range(grid[0]):
                    for y in builtins.range(grid[1]):
                        I.interpreter_builder.set_grid_idx(x, y, 0)
                        barrier[0] = threading.Barrier(2)
                        errors = []

                        def body(sid):
                            state.sid = sid
                            try:
                                self.fn(**args)
                            except Exception as ex:  # surface the first failure
                                errors.append(ex)
                                barrier[0].abort()

                        ts = [threading.Thread(target=body, args=(i,)) for i in (0, 1)]
                        for t in ts:
                            t.start()
                        for t in ts:
                            t.join()
                        if errors:
                            raise errors[0]
            finally:
                scope.restore()
            self._restore_args_dev(args_dev, args_hst, kwargs, kwargs_hst)

    class Launcher:
        def __init__(self, kernel):
            self.kernel = kernel

        def __getitem__(self, grid):
            def launch(**kw):
                for e in extra:
                    kw.pop(e, None)
                return TwoSubCoreExecutor(self.kernel.rewrite(), self.kernel.arg_names, grid)(**kw)
            return launch

    for name in ("_attn_fwd", "_attn_bwd_dq_dsink", "_attn_bwd_dk_dv"):
        setattr(SFA, name, Launcher(getattr(SFA, name)))

    def scalar_range(*a):
        for i in builtins.range(*a):
            yield scalar(i)
    SFA.range = scalar_range

    orig_cast = I.InterpreterBuilder.cast_impl

    def cast(self, src, dst_type):
        s, d = src.dtype.scalar, dst_type.scalar
        if (s != d and (s == tl.bfloat16 or d == tl.bfloat16) and s != tl.float32 and d != tl.float32
                and s.is_floating() and d.is_floating()):
            return orig_cast(self, orig_cast(self, src, tl.float32), dst_type)
        return orig_cast(self, src, dst_type)
    I.InterpreterBuilder.cast_impl = cast

    orig_dot = I.InterpreterBuilder.create_dot

    def dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        def up(x):
            if x.dtype.scalar == tl.bfloat16:
                return I.TensorHandle(I._convert_float(x.data, tl.bfloat16, tl.float32, None).view(np.float32),
                                      tl.float32)
            return x
        return orig_dot(self, up(a), up(b), d, input_precision, max_num_imprecise_acc)
    I.InterpreterBuilder.create_dot = dot

    def arange(self, start, end, *, ret_ty=None):
        start, end = int(start), int(end)
        if ret_ty is None:
            ret_ty = tl.block_type(tl.int32, [end - start])
        return self.tensor(self.builder.create_make_range(ret_ty, start, end), ret_ty)
    SEM.TritonSemantic.arange = arange

    def validate_block_shape(shape):
        n = 1
        for s in shape:
            n *= int(s)
        return n
    CORE.validate_block_shape = validate_block_shape
    return SFA


def run_reference(SFA, q, kv, sink, idx, scale, do):
    """Forward + backward through the reference autograd op.

    Returns (out, lse2, dq, dkv, dsink) where lse2 is the reference's saved base-2
    log-sum-exp (captured from its first ``torch.empty`` allocation, ``SFA.py:107``).
    """
    import torch
    qr = q.clone().requires_grad_()
    kvr = kv.clone().requires_grad_()
    sr = sink.clone().requires_grad_()
    captured = []
    real_empty = torch.empty

    def spy_empty(*a, **k):
        t = real_empty(*a, **k)
        captured.append(t)
        return t
    torch.empty = spy_empty
    try:
        out = SFA.SparseFlashAttentionTriton.apply(qr, kvr, sr, idx, scale)
    finally:
        torch.empty = real_empty
    lse2 = captured[0].clone()
    out.backward(do)
    return out.detach(), lse2, qr.grad.detach(), kvr.grad.detach(), sr.grad.detach()
