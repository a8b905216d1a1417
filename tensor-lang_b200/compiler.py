"""``TensorCompiler`` facade with the reference's constructor and entry point.

``tensorlang/compiler.py:30-42, 858``: ``TensorCompiler(debug_mode, debug_info,
debug_ast, cache_layers, transpile).compile_and_execute(path)``.  Parsing and
type checking are the reference frontend's (``tensorlang.lark``,
``ast_builder.build_ast``, ``type_checker.type_checker``), imported from the
``tensorlang`` package the caller already has; execution is ``Program``.
With ``cache_layers`` every result is written to ``cache/<path>/<name>.npy``
and top-level gradients to ``<name>.grad.npy``, the layout the reference's test
runner reads (compiler.py:682-684, 1610-1612).
"""
from __future__ import annotations

import contextlib
import io
from pathlib import Path
from typing import Dict, Optional

import numpy as np

from .engine import Program


def parse_program(path: str, grammar: Optional[str] = None):
    """Parse and type-check a .tl file with the reference frontend."""
    from lark import Lark  # the reference's parser dependency
    import tensorlang  # noqa: F401  (the reference package)
    from tensorlang.ast_builder import build_ast
    from tensorlang.type_checker import type_checker

    if grammar is None:
        cands = [Path("tensorlang.lark"), Path(tensorlang.__file__).resolve().parent.parent / "tensorlang.lark"]
        grammar = next((str(c) for c in cands if c.exists()), None)
        if grammar is None:
            raise FileNotFoundError("tensorlang.lark not found next to the tensorlang package")
    parser = Lark(Path(grammar).read_text(), start="program", parser="lalr")
    with contextlib.redirect_stdout(io.StringIO()):
        tree = parser.parse(Path(path).read_text())
        ast, _out, _fns = build_ast(tree, False, False)
        ok, env = type_checker(ast, {}, False, False)
    if not ok:
        raise TypeError(f"{path} does not type-check")
    return ast, env


class TensorCompiler:
    def __init__(self, debug_mode=False, debug_info=False, debug_ast=False, cache_layers=False,
                 transpile=False, device: int = 0):
        if transpile:
            raise NotImplementedError("--transpile (WGSL/WebGPU) is not part of this backend")
        self.debug_mode = debug_mode
        self.cache_layers = cache_layers
        self.device = device
        self.results: Dict[str, np.ndarray] = {}

    def compile_and_execute(self, tensorlang_file: str) -> Dict[str, np.ndarray]:
        ast, env = parse_program(tensorlang_file)
        cache_dir = Path("cache") / tensorlang_file
        prog = Program(ast, env, device=self.device, save_dir=str(cache_dir))
        self.results = prog.run()
        if self.cache_layers:
            cache_dir.mkdir(parents=True, exist_ok=True)
            for name, arr in self.results.items():
                np.save(cache_dir / f"{name}.npy", arr)
        prog.free()
        return self.results
