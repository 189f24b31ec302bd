"""``bitcache._C`` (the reference's torch extension, src/torch_binding.cpp:17-177):
the operators of ``bitcache_b200._C``."""
from bitcache_b200._C import *  # noqa: F401,F403
from bitcache_b200._C import __all__  # noqa: F401
