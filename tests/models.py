"""Test helpers: the seeded synthetic models live in oracle/models.py."""
from oracle.models import ModelWeights, prompt, rel  # noqa: F401
