"""Built-in metric modules."""
