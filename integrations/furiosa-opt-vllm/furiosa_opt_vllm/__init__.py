"""vLLM platform plugin: vLLM keeps its scheduler, sampling parameters and OpenAI-compatible API;
every forward pass runs through the B200 engine (``furiosa_opt_engine``).

The entry point is declared under ``vllm.platform_plugins`` (pyproject.toml, and the metadata
directory beside this package for use from a source tree on ``sys.path``).
"""


def register() -> str:
    # vLLM calls this while it resolves its platform; importing vLLM here would cycle.
    return "furiosa_opt_vllm.platform.B200Platform"
