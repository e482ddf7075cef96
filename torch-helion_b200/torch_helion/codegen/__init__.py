"""Codegen: per-kernel B200 launch plans (emit_program)."""

from .emit import CodegenError, emit_program

__all__ = ["CodegenError", "emit_program"]
