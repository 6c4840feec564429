"""B200-native (sm_100a) forward of the Laya decision classifier, exposed as
the ``b200`` mode of the reference engine contract.

Public entry points: ``create_engine(mode="b200", ...)``, ``B200Engine``,
``B200Dispatcher`` (request-parallel over several GPUs) and the weight /
workload helpers.
"""
from .config import LAYA, TINY, LayaConfig
from .modes import create_engine, MODES

__all__ = ["LAYA", "TINY", "LayaConfig", "create_engine", "MODES"]
