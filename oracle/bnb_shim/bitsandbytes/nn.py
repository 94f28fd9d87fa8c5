"""Empty: no upstream ``Experts4bit`` so the reference picks its vendored classes."""
