"""Built-in benchmark modules."""
