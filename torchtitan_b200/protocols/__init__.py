from .model import BaseModel, BaseModelArgs
from .model_spec import ModelSpec
from .model_converter import ModelConverter, ModelConvertersContainer
from .state_dict_adapter import BaseStateDictAdapter, StateDictAdapter

__all__ = [
    "BaseModel",
    "BaseModelArgs",
    "ModelSpec",
    "ModelConverter",
    "ModelConvertersContainer",
    "BaseStateDictAdapter",
    "StateDictAdapter",
]
