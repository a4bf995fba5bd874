"""SGLang plugin: SGLang keeps its scheduler, radix cache and OpenAI-compatible server; every
forward batch runs through the B200 engine. SGLang discovers the platform and the worker hooks
through package entry points (pyproject.toml)."""


def activate() -> str:
    """The platform class path for the ``sglang.srt.platforms`` entry point."""
    return "furiosa_opt_sglang.platform.Platform"


def register() -> None:
    """Installs the model-runner hook at SGLang startup (``sglang.srt.plugins``)."""
    from furiosa_opt_sglang.hooks import register as install

    install()
