/* Embeds the sm_100a cubin built from csrc/kernels/kernels.cu into the
 * shared library; F4S_KERNEL_IMAGE is its path, set by the build. */
    .section .rodata
    .global f4s_kernel_image_begin
    .global f4s_kernel_image_end
    .balign 256
f4s_kernel_image_begin:
    .incbin F4S_KERNEL_IMAGE
f4s_kernel_image_end:
    .byte 0
    .section .note.GNU-stack,"",@progbits
