"""``bitcache.functional`` (reference bitcache/functional.py:17-139): the entry
points of ``bitcache_b200.functional``."""
from bitcache_b200.functional import *  # noqa: F401,F403
from bitcache_b200.functional import __all__  # noqa: F401
