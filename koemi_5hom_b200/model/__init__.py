from koemi_5hom_b200.model.network import ExecutionMode, HermBlock, KoemiModel, KoemiOutput, RouterStatistics
from koemi_5hom_b200.model.settings import PAD_TOKEN_ID, ModelSettings
from koemi_5hom_b200.model.state import KOEMI_STATE_FIELDS, KoemiState, LayeredKoemiState

__all__ = ["ExecutionMode", "HermBlock", "KOEMI_STATE_FIELDS", "KoemiModel", "KoemiOutput", "KoemiState",
           "LayeredKoemiState", "ModelSettings", "PAD_TOKEN_ID", "RouterStatistics"]
