from .model_registry import ModelRegistry, ModelSpec
from .task_registry import TaskRegistry
from .task_adapter import TaskAdapter

__all__ = ["ModelRegistry", "ModelSpec", "TaskRegistry", "TaskAdapter"]
