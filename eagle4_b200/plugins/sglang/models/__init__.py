"""Draft architectures SGLang's model registry loads from this package (``EntryClass`` per module)."""
