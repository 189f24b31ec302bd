"""The reference's import name: ``import bitcache`` gives this repository's
B200 implementation (package ``bitcache_b200``) under the names the reference
exposes (bitcache/__init__.py and bitcache/functional.py of anishesg/bitcache):
``bitcache.BitCache``, ``bitcache.functional``, ``bitcache._C`` and
``bitcache._require_extension``.  Nothing else lives here.
"""
from bitcache_b200 import BitCache, _require_extension  # noqa: F401

from . import _C, functional  # noqa: E402,F401

__all__ = ["BitCache", "functional", "_C", "_require_extension"]


def __getattr__(name: str):
    if name == "_HAS_EXTENSION":
        import bitcache_b200

        return bitcache_b200._HAS_EXTENSION
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
