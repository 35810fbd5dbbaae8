"""Launch, timing and measurement helpers."""
