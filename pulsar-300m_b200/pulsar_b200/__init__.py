"""pulsar_b200: B200-native (sm_100a) KV-cache decode engine for the Pulsar-283M model."""

from .config import PulsarConfig, engine_supported  # noqa: F401

__all__ = ["PulsarConfig", "engine_supported"]
