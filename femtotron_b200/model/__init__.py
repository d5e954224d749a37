"""Alias of :mod:`femtotron_b200.models` under the reference's singular package name."""
from femtotron_b200.models import *  # noqa: F401,F403
from femtotron_b200.models import __all__  # noqa: F401
