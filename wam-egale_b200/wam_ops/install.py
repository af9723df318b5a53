"""Drop-in installer: run a model's Wan blocks on the B200 native path.

Same surface and preconditions as the reference installer
(算子研究/wam_ops/install.py:5-61): `install_block` is a context manager
that swaps the block's (and its two attentions') classes, binds a
NativeBlock, and restores everything on exit; `install_model` does it for
every block of `model.blocks`. Only the instance passed in is modified.

Both reference implementation names are accepted and run the same single
B200 path ("baseline" keeps the reference's rule that it takes no
optimisation flags); `execution_mode` is validated and otherwise has no
effect, because there is one code path.
"""
from contextlib import ExitStack, contextmanager


@contextmanager
def install_block(block, implementation="baseline", *, execution_mode=None, fused_ffn1=None):
    from .block import Attention, TransformerBlock
    from .native import NativeBlock

    if implementation not in ("baseline", "optimized"):
        raise ValueError("implementation must be 'baseline' or 'optimized'")
    if block.attn_mode != "torch":
        raise ValueError("the original Torch attention mode is required as the matching baseline")
    modules = (block, block.attn1, block.attn2)
    if any("forward" in module.__dict__ for module in modules):
        raise ValueError("the model carries experimental forward overrides; cannot install")
    if any(attention.cache_mode != "original" for attention in modules[1:]):
        raise ValueError("only the original KV protocol is supported")
    if implementation == "baseline" and (execution_mode is not None or fused_ffn1 is not None):
        raise ValueError("baseline is frozen; optimization flags are invalid")
    if execution_mode not in (None, "sequential", "tiled", "persistent"):
        raise ValueError("mode must be sequential, tiled or persistent")
    classes = tuple(type(module) for module in modules)
    operations = tuple(getattr(attention, "attn_op", None) for attention in modules[1:])
    previous_native = block.__dict__.get("_native_block")
    try:
        for module, kind in zip(modules, (TransformerBlock, Attention, Attention)):
            module.__class__ = kind
        native = NativeBlock(block, fused_ffn1=bool(fused_ffn1), mode=execution_mode or "sequential")
        object.__setattr__(block, "_native_block", native)
        yield block
    finally:
        for module, kind in zip(modules, classes):
            module.__class__ = kind
        for attention, operation in zip(modules[1:], operations):
            if operation is not None:
                attention.attn_op = operation
        if previous_native is None:
            block.__dict__.pop("_native_block", None)
        else:
            object.__setattr__(block, "_native_block", previous_native)


@contextmanager
def install_model(model, implementation="baseline", **options):
    with ExitStack() as stack:
        for block in model.blocks:
            stack.enter_context(install_block(block, implementation, **options))
        yield model
