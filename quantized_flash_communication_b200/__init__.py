"""quantized_flash_communication_b200: B200-native quantized tensor-parallel communication.
"""
__version__ = "0.1.0"
