"""Framework adapters for the B200 backend (mirrors the reference's ``integrations`` package)."""
