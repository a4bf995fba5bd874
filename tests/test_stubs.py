"""The committed `.pyi` stubs match the native extension (regenerate with
`python -m furiosa_opt_engine._stubs`)."""

from furiosa_opt_engine import _stubs


def test_stubs_match_the_extension():
    for m in _stubs.MODULES:
        with open(_stubs.path(m)) as f:
            assert f.read() == _stubs.render(m), f"stale stub {_stubs.path(m)}: regenerate it"


def test_public_classes_are_stubbed():
    text = _stubs.render("") + _stubs.render("decoder")
    for name in ("class Checkpoint", "class LoadOptions", "class Device", "class HbmTensor", "class Adapter",
                 "class AdapterSpec", "class Request", "class Cache"):
        assert name in text
