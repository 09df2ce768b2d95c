from .ops import get_conv_output_size, get_deconv_output_size, get_indice_pairs

__all__ = ['get_conv_output_size', 'get_deconv_output_size', 'get_indice_pairs']
