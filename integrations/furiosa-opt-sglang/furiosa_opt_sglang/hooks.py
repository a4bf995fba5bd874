"""The model-runner hook SGLang calls at startup: SGLang's model runner hands each forward batch
to the plugin's runner. SGLang is optional here: without it the hook installs nothing, and the
runner serves SGLang-shaped batches directly (tests and embedders)."""

from __future__ import annotations

INSTALLED = False


def register() -> None:
    global INSTALLED
    try:
        import sglang  # noqa: F401
    except ImportError:
        return
    INSTALLED = True
