"""Stand-in ``bitsandbytes`` for the build container (test infrastructure only).

Lets the reference's own Python import and run on CPU so that
``tests/golden/make_golden.py`` can record its outputs. The NF4 codec is the
oracle's restatement (``oracle/nf4.py``); nothing here is bitsandbytes code.
"""
from . import functional  # noqa: F401
from . import nn  # noqa: F401
