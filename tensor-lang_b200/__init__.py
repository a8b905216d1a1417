"""tensor_lang_b200 -- B200 (sm_100a) execution backend for TensorLang programs.

Drop-in for the execution half of the reference (davro/tensor-lang):
``KernelGenerator`` keeps the per-op lowering interface of
``tensorlang/kernel_generator.py``; ``Program`` executes a lowered program
(the reference frontend's AST and type environment) on one GPU through
libtlb200.so; ``TensorCompiler`` mirrors ``tensorlang/compiler.py``'s
``TensorCompiler.compile_and_execute`` on top of them; ``dp`` runs a training
loop data-parallel over several GPUs with NCCL.
"""
from .runtime import Device, TLCudaError, load_library, launch_count  # noqa: F401
from .kernel_generator import KernelGenerator  # noqa: F401
from .engine import Program, lower_let  # noqa: F401
from .compiler import TensorCompiler  # noqa: F401
from . import programs  # noqa: F401

__version__ = "0.1.0"
