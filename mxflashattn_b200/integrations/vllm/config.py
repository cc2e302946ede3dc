"""vLLM version pin of the integration contract (integrations/vllm/config.py:1-11).

The reference validated its hook against vLLM 0.17.0; the same pin and error
text are kept so callers that check it behave identically.
"""

VLLM_TARGET_VERSION = "0.17.0"


def validate_vllm_version(version: str) -> None:
    if version != VLLM_TARGET_VERSION:
        raise RuntimeError(
            f"MXFlashAttn currently targets vLLM {VLLM_TARGET_VERSION}; found {version}. "
            "Confirm compatibility before selecting an attention backend."
        )
