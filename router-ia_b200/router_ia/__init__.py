"""router-ia attention hot path on B200 kernels.

This package directory only provides ``router_ia.qwen36_attention_cache``.
``extend_path`` lets it share the ``router_ia`` namespace with an existing
router-ia install placed after it on ``sys.path``: every other module
(``qwen36_chat_batch``, ``qwen36_cached_loop`` ...) then resolves to that
install, and their ``from . import qwen36_attention_cache`` resolves here.
"""

from pkgutil import extend_path

__path__ = extend_path(__path__, __name__)

__version__ = "0.1.0"
