"""Worker-side step driver and step messages."""
