from .sample import IGNORE_INDEX, VARLEN_TOKEN_STAT_NAMES, PreparedVarlenPack, RLSample

__all__ = ["IGNORE_INDEX", "VARLEN_TOKEN_STAT_NAMES", "PreparedVarlenPack", "RLSample"]
