"""Run the reference emulator (bkase/gbxcule) from its own source on the host.

TEST INFRASTRUCTURE ONLY. This module is the golden-vector generator; it is
never imported by the product package, the GPU tests or the benchmark.

The reference's hot path is Warp-DSL Python: ``cpu_step_builder.py`` splices
instruction templates into a kernel skeleton with libcst and Warp JIT-compiles
it. Neither ``warp-lang`` nor ``libcst`` is installable here, so this module
supplies the two missing pieces and nothing else:

* ``_FakeWarp``: a host-side model of the Warp runtime subset the reference
  uses (typed casts, ``where``, arrays, ``launch``/``copy``/``zeros``).  Arrays
  are ``bytearray`` (u8) or ``array.array`` (i32 'i', i64 'q', f32 'f'), so a
  store outside the element type's range raises instead of wrapping, and every
  value the kernel computes is an exact Python int. ``wp.where(c, a, b)`` is
  numpy-ordered (a if c else b) as in warp-lang 1.11 (the version the
  reference's lockfile pins).
* ``_assemble_kernel``: the libcst splice of ``build_cpu_step_source``
  (``cpu_step_builder.py:1786-1856``) redone with the stdlib ``ast`` module:
  placeholder renaming as ``TemplateSpecializer`` (``:26-38``), the two-level
  bucket dispatch of ``_build_bucket_dispatch`` (``:92-125``) and injection at
  ``INSTRUCTION_DISPATCH``/``CB_DISPATCH``/``POST_STEP_DISPATCH``.

Everything else - the skeleton text, the templates, the ISA table, the
template map, constants, the backend's reset/step/readback code, the renderer
and the reset-cache kernels - is the reference's own code, imported from the
tree given by ``load_reference(path)``.
"""

from __future__ import annotations

import array
import ast
import importlib
import inspect
import sys
import textwrap
import types
from pathlib import Path

import numpy as np

# ---------------------------------------------------------------------------
# Warp runtime model
# ---------------------------------------------------------------------------

_I32 = (1 << 31)


def _int32(x):
    x = int(x)
    return ((x + _I32) & 0xFFFFFFFF) - _I32


def _int64(x):
    x = int(x)
    return ((x + (1 << 63)) & 0xFFFFFFFFFFFFFFFF) - (1 << 63)


def _uint8(x):
    return int(x) & 0xFF


def _float32(x):
    return np.float32(x)


class FakeArray:
    """A 1-D device array stand-in; ``data`` is what kernels index."""

    def __init__(self, data, dtype):
        self.data = data
        self.dtype = dtype

    def __len__(self):
        return len(self.data)

    def numpy(self):
        if isinstance(self.data, bytearray):
            return np.frombuffer(self.data, dtype=np.uint8)
        return np.frombuffer(self.data, dtype={"i": np.int32, "q": np.int64, "f": np.float32}[self.data.typecode])

    def assign(self, values):
        self.numpy()[:] = np.asarray(values).reshape(-1)

    @property
    def shape(self):
        return (len(self.data),)


def _make_container(n, dtype):
    if dtype is _uint8:
        return bytearray(n)
    code = {_int32: "i", _int64: "q", _float32: "f"}[dtype]
    return array.array(code, bytes(n * array.array(code).itemsize))


class _FakeWarp(types.ModuleType):
    """Module object installed as ``warp`` while the reference runs."""

    def __init__(self):
        super().__init__("warp")
        self.uint8 = _uint8
        self.int32 = _int32
        self.int64 = _int64
        self.float32 = _float32
        self.config = types.SimpleNamespace(mode=None)
        self._tid = 0

    # decorators / annotations
    @staticmethod
    def func(f):
        return f

    @staticmethod
    def kernel(f):
        return f

    @staticmethod
    def where(cond, a, b):
        return a if cond else b

    def tid(self):
        return self._tid

    # runtime
    def init(self):
        return None

    def get_device(self, name):
        return name

    def synchronize(self):
        return None

    def array(self, data=None, dtype=None, device=None, **_kw):
        if data is None:  # used as a type annotation: wp.array(dtype=...)
            return None
        np_dtype = {_uint8: np.uint8, _int32: np.int32, _int64: np.int64, _float32: np.float32}[dtype]
        src = np.ascontiguousarray(np.asarray(data, dtype=np_dtype).reshape(-1))
        arr = FakeArray(_make_container(src.size, dtype), dtype)
        arr.numpy()[:] = src
        return arr

    def zeros(self, n, dtype=None, device=None, **_kw):
        return FakeArray(_make_container(int(n), dtype), dtype)

    def empty(self, n, dtype=None, device=None, **_kw):
        return self.zeros(n, dtype=dtype, device=device)

    def copy(self, dest, src, dest_offset=0, src_offset=0, count=None):
        d, s = dest.numpy(), src.numpy()
        if count is None:
            count = min(len(d) - dest_offset, len(s) - src_offset)
        d[dest_offset:dest_offset + count] = s[src_offset:src_offset + count]

    def launch(self, kernel, dim, inputs, device=None, **_kw):
        args = [x.data if isinstance(x, FakeArray) else x for x in inputs]
        for t in range(int(dim)):
            self._tid = t
            kernel(*args)


def _install_stubs():
    # One model per process: reference modules bind ``wp`` at import time, so
    # a second instance would leave launches and kernels on different objects.
    wp = sys.modules.get("warp")
    if isinstance(wp, _FakeWarp):
        return wp
    wp = _FakeWarp()
    sys.modules["warp"] = wp
    cst = types.ModuleType("libcst")
    cst.CSTTransformer = object  # only subclassed at import; never used
    sys.modules["libcst"] = cst
    return wp


# ---------------------------------------------------------------------------
# ast-based kernel assembly (replaces the libcst splice)
# ---------------------------------------------------------------------------

class _Rename(ast.NodeTransformer):
    def __init__(self, repl):
        self.repl = repl

    def visit_Name(self, node):
        new = self.repl.get(node.id)
        if new is not None:
            return ast.copy_location(ast.Name(id=new, ctx=node.ctx), node)
        return node


def _template_body(func, repl):
    src = textwrap.dedent(inspect.getsource(func))
    fdef = ast.parse(src).body[0]
    assert isinstance(fdef, ast.FunctionDef)
    body = [_Rename(dict(repl or {})).visit(stmt) for stmt in fdef.body]
    # drop a leading docstring expression (harmless either way)
    if body and isinstance(body[0], ast.Expr) and isinstance(getattr(body[0], "value", None), ast.Constant):
        body = body[1:] or [ast.Pass()]
    return body


def _eq(var, val):
    return ast.Compare(left=ast.Name(id=var, ctx=ast.Load()), ops=[ast.Eq()],
                       comparators=[ast.Constant(value=val)])


def _linear(specs, default_body, var):
    node = default_body
    for spec in reversed(specs):
        node = [ast.If(test=_eq(var, spec.opcode), body=_template_body(spec.template, spec.replacements),
                       orelse=node)]
    return node


def _bucket(specs, default_body, var, hi_var):
    buckets = {}
    for spec in specs:
        buckets.setdefault(spec.opcode >> 4, []).append(spec)
    node = default_body
    for hi in sorted(buckets, reverse=True):
        inner = _linear(sorted(buckets[hi], key=lambda s: s.opcode), default_body, var)
        node = [ast.If(test=_eq(hi_var, hi), body=inner, orelse=node)]
    return node


class _Inject(ast.NodeTransformer):
    def __init__(self, table):
        self.table = table
        self.inside = False

    def visit_FunctionDef(self, node):
        if node.name != "cpu_step":
            return node
        self.generic_visit(node)
        return node

    def _splice(self, stmts):
        out = []
        for s in stmts:
            if isinstance(s, ast.Expr) and isinstance(s.value, ast.Name) and s.value.id in self.table:
                out.extend(self.table[s.value.id])
            else:
                out.append(self.visit(s))
        return out or [ast.Pass()]

    def generic_visit(self, node):
        for field in ("body", "orelse", "finalbody"):
            stmts = getattr(node, field, None)
            if isinstance(stmts, list) and stmts and isinstance(stmts[0], ast.stmt):
                setattr(node, field, self._splice(stmts))
        return node


def _make_builder(builder_mod):
    def build_cpu_step_kernel(opcode_templates, default_template, constants, *,
                              cb_opcode_templates=None, cb_default_template=None,
                              post_step_body=None):
        default_body = _template_body(default_template.template, default_template.replacements)
        cb_default = cb_default_template or default_template
        cb_default_body = _template_body(cb_default.template, cb_default.replacements)
        table = {
            "INSTRUCTION_DISPATCH": _bucket(list(opcode_templates), default_body, "opcode", "opcode_hi"),
            "CB_DISPATCH": _bucket(list(cb_opcode_templates or ()), cb_default_body, "cb_opcode", "cb_opcode_hi"),
            "POST_STEP_DISPATCH": list(post_step_body or []),
        }
        src = builder_mod._CPU_STEP_SKELETON.format(**constants)
        tree = _Inject(table).visit(ast.parse(src))
        ast.fix_missing_locations(tree)
        mod = types.ModuleType("gbxcule_ref_cpu_step")
        exec(compile(tree, "<reference cpu_step>", "exec"), mod.__dict__)
        return mod.cpu_step

    def get_template_body(func_obj, replacements=None):
        return _template_body(func_obj, replacements)

    return build_cpu_step_kernel, get_template_body


# ---------------------------------------------------------------------------
# Loader
# ---------------------------------------------------------------------------

class Reference:
    """Handles to the reference modules running under the Warp model."""

    def __init__(self, wp, modules):
        self.wp = wp
        self.m = modules

    def backend(self, rom_path: str, *, num_envs: int, frames_per_step: int,
                release_after_frames: int, stage: str = "obs_only",
                render_pixels: bool = False, render_pixels_packed: bool = False,
                render_bg: bool = False):
        cls = self.m["warp_vec"].WarpVecCpuBackend
        return cls(rom_path, num_envs=num_envs, frames_per_step=frames_per_step,
                   release_after_frames=release_after_frames, stage=stage,
                   render_pixels=render_pixels, render_pixels_packed=render_pixels_packed,
                   render_bg=render_bg, render_on_step=False)

    def launch_step(self, be, actions: np.ndarray, render: bool = False) -> None:
        """``step_torch`` semantics: no host range check, one kernel launch
        (plus the env-0 BG frame render when ``render`` and ``render_bg``)."""
        be._actions.assign(np.asarray(actions, dtype=np.int32))
        be._launch_step(be._actions, render=render)

    def frame_bg(self, be) -> np.ndarray:
        """The env-0 160x144 BG shade frame (``read_frame_bg_shade_env0``)."""
        return np.frombuffer(be.read_frame_bg_shade_env0(), dtype=np.uint8).copy()

    def render_packed(self, be) -> np.ndarray:
        k = self.m["ppu"].ppu_render_shades_downsampled_packed_all_envs
        out = self.wp.zeros(be.num_envs * 1440, dtype=_uint8)
        self.wp.launch(k, dim=be.num_envs * 1440, inputs=[be._mem, out, 0])
        return out.numpy().reshape(be.num_envs, 72, 20).copy()

    def render_shades(self, be) -> np.ndarray:
        k = self.m["ppu"].ppu_render_shades_downsampled_all_envs
        out = self.wp.zeros(be.num_envs * 5760, dtype=_uint8)
        self.wp.launch(k, dim=be.num_envs * 5760, inputs=[be._mem, out])
        return out.numpy().reshape(be.num_envs, 72, 80).copy()

    def reset_cache(self, be, env_idx: int = 0):
        return self.m["reset_cache"].ResetCache.from_backend(be, env_idx=env_idx)

    def apply_mask_kernels(self, cache, mask: np.ndarray) -> None:
        """The CUDA restore path (``_launch_masked_copies``) on the model."""
        mask_wp = self.wp.array(np.asarray(mask, dtype=np.uint8), dtype=_uint8)
        cache._launch_masked_copies(mask_wp)


def load_reference(ref_root: str | Path, boot_path: str | Path) -> Reference:
    """Import the reference package from ``ref_root/src`` under the model."""
    ref_root = Path(ref_root)
    wp = _install_stubs()
    src = str(ref_root / "src")
    if src not in sys.path:
        sys.path.insert(0, src)
    import os
    os.environ["GBXCULE_SKIP_WARP_WARMUP"] = "1"
    for var in ("GBXCULE_TRAP_RST38", "GBXCULE_TRAP_PC", "GBXCULE_MAX_INSTR", "GBXCULE_WATCH_ADDR"):
        os.environ.pop(var, None)
    builder = importlib.import_module("gbxcule.kernels.cpu_step_builder")
    cpu_step = importlib.import_module("gbxcule.kernels.cpu_step")
    build_fn, body_fn = _make_builder(builder)
    cpu_step.build_cpu_step_kernel = build_fn
    cpu_step.get_template_body = body_fn
    warp_vec = importlib.import_module("gbxcule.backends.warp_vec")
    warp_vec.BOOTROM_PATH = Path(boot_path)
    mods = {
        "builder": builder,
        "cpu_step": cpu_step,
        "warp_vec": warp_vec,
        "ppu": importlib.import_module("gbxcule.kernels.ppu_render_downsampled"),
        "reset_cache": importlib.import_module("gbxcule.core.reset_cache"),
        "isa": importlib.import_module("gbxcule.core.isa_sm83"),
        "cartridge": importlib.import_module("gbxcule.core.cartridge"),
    }
    return Reference(wp, mods)
