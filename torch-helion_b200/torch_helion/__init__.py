"""torch-helion on B200: the torch-helion front end (capture, OpGraph,
optimizer, planner) with hand-written sm_100a kernels as the backend."""

from .artifact import load_compiled
from .config import CompileConfig
from .pipeline import CompileResult, compile_model

__version__ = "0.1.0.dev0+b200"

__all__ = ["CompileConfig", "CompileResult", "compile_model", "load_compiled", "__version__"]
