"""Request-scoped attention context (the role of the native engine's ContextVars,
model/kernels.py:37-120, 643-757).

A serving process owns one model graph and runs many requests through it, so the
per-request facts the sparse attention needs -- the packed text/audio prefix
length, the generated video's geometry, a request-level sparse budget -- are not
constructor arguments but context variables set around each request:

    with attention_protected_prefix(prefix_tokens), attention_video_layout(frames, frame_tokens):
        block(...)

The B200 backends read them through a *context source*: any object with the
getter functions below.  This module is the default source; an engine that
already keeps these ContextVars (the reference's model/kernels.py has the same
three getters) passes its own module as `context=` so both read one state.
"""

from __future__ import annotations

from contextlib import contextmanager
from contextvars import ContextVar

_SPARSE_TOPK: ContextVar[float | None] = ContextVar("h3b_attention_sparse_topk", default=None)
_PROTECTED_PREFIX: ContextVar[int] = ContextVar("h3b_attention_protected_prefix", default=0)
_VIDEO_LAYOUT: ContextVar[tuple[int, int] | None] = ContextVar("h3b_attention_video_layout", default=None)
_VIDEO_GRID: ContextVar[tuple[int, int] | None] = ContextVar("h3b_attention_video_grid", default=None)


def current_attention_protected_prefix() -> int:
    """Packed text / reference / audio prefix length of the current request (0: none)."""
    return int(_PROTECTED_PREFIX.get())


def current_attention_video_layout() -> tuple[int, int] | None:
    """(latent frames, tokens per frame) of the generated video rows, or None."""
    return _VIDEO_LAYOUT.get()


def current_attention_video_grid() -> tuple[int, int] | None:
    """(patch rows, patch columns) of one latent frame, or None."""
    return _VIDEO_GRID.get()


def current_attention_sparsity() -> float | None:
    """Request-level sparse Top-K budget, or None for dense attention."""
    return _SPARSE_TOPK.get()


@contextmanager
def attention_sparsity(topk: float | None):
    """Select dense (None) or a request-scoped sparse budget in [0.5, 1.0]
    (model/kernels.py:666-676)."""
    if topk is not None and not 0.5 <= topk <= 1.0:
        raise ValueError("attention sparse topk must be between 0.5 and 1.0")
    token = _SPARSE_TOPK.set(None if topk is None else float(topk))
    try:
        yield
    finally:
        _SPARSE_TOPK.reset(token)


@contextmanager
def attention_protected_prefix(token_count: int):
    """Expose the packed conditioning prefix length (model/kernels.py:706-716)."""
    if token_count < 0:
        raise ValueError("attention protected prefix cannot be negative")
    token = _PROTECTED_PREFIX.set(int(token_count))
    try:
        yield
    finally:
        _PROTECTED_PREFIX.reset(token)


@contextmanager
def attention_video_layout(latent_frames: int, frame_tokens: int, *, grid_height: int | None = None,
                           grid_width: int | None = None):
    """Expose the generated video's frame-major geometry (model/kernels.py:719-754)."""
    if latent_frames <= 0 or frame_tokens <= 0:
        raise ValueError("attention video layout dimensions must be positive")
    if (grid_height is None) != (grid_width is None):
        raise ValueError("attention video grid requires both height and width")
    if grid_height is not None:
        if grid_height <= 0 or grid_width is None or grid_width <= 0:
            raise ValueError("attention video grid dimensions must be positive")
        if int(grid_height) * int(grid_width) != int(frame_tokens):
            raise ValueError("attention video grid does not match tokens per frame")
    token = _VIDEO_LAYOUT.set((int(latent_frames), int(frame_tokens)))
    grid_token = _VIDEO_GRID.set(None if grid_height is None else (int(grid_height), int(grid_width)))
    try:
        yield
    finally:
        _VIDEO_GRID.reset(grid_token)
        _VIDEO_LAYOUT.reset(token)


def source_getter(source, name: str, default):
    """`source.name()` if the context source has that getter, else `default`."""
    fn = getattr(source, name, None)
    return fn() if callable(fn) else default
