"""Drop-in for the reference's ``bench/attention.py`` (the attention backend registry).

Only ``bench.attention`` is provided here. The package path is extended with every other
``bench`` directory on ``sys.path``, so with the reference checked out beside this one its
own ``bench.attention_bench``, ``bench.decode_ncu`` and ``bench.harness`` still import, and
import this ``bench.attention``.
"""

import pkgutil

__path__ = pkgutil.extend_path(__path__, __name__)
