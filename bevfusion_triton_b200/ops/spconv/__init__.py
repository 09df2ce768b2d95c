from .ops import (fused_indice_conv, get_conv_output_size, get_deconv_output_size, get_indice_pairs, indice_conv,
                  indice_conv_backward, indice_maxpool, indice_maxpool_backward)

__all__ = ['fused_indice_conv', 'get_conv_output_size', 'get_deconv_output_size', 'get_indice_pairs', 'indice_conv',
           'indice_conv_backward', 'indice_maxpool', 'indice_maxpool_backward']
