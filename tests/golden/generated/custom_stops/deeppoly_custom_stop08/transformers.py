import gc
import json
import os
import torch
import operator
from constraintflow.lib.globals import device_mode
from constraintflow.lib.polyexp import PolyExpSparse
from constraintflow.lib.symexp import *
from constraintflow.gbcsr.sparse_tensor import SparseTensor
from constraintflow.lib.llist import Llist
from constraintflow.gbcsr.tensor_ops import *
class deeppoly:
	def Affine(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_24 = prev.dot(curr.get_metadata('weight', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), abs_elem.get_poly_size(), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1, mats_input = 'rhs')
		cse_var_23 = repeat(curr.get_metadata('bias', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_67 = cse_var_24.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_44 = PolyExpSparse(abs_elem.network, cse_var_67 , binary(cse_var_24.get_const(), cse_var_23, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_105 = binary(get_dims(cse_var_67, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), 1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_13 = repeat((binary(curr.get_metadata('layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), SparseTensor([], [], 0, torch.tensor([]), dense_const=8, type= type(8)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([1, curr_size])), operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_108 = Llist(abs_elem.network, [1]*(cse_var_105), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist()).get_metadata('layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_11 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size]))
		cse_var_107 = Llist(abs_elem.network, [1]*(cse_var_105), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_112 = binary(repeat(cse_var_108, torch.tensor([1, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_13, operator.lt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_111 = unary(cse_var_108, operator.neg, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_109 = abs_elem.get_elem('L', cse_var_107, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_110 = abs_elem.get_elem('U', cse_var_107, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_115 = cse_var_110.get_const()
		cse_var_114 = cse_var_110.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_117 = cse_var_109.get_const()
		cse_var_116 = cse_var_109.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		phi_trav_exp1_1_1 = cse_var_44
		while_iteration = -1
		while(True):
			while_iteration += 1
			cse_var_27 = phi_trav_exp1_1_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			vertices1_1_1 = binary(cse_var_27, cse_var_11, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop_default1 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			cse_var_113 = repeat(cse_var_112, torch.tensor([batch_size, 1, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop_temp1 = binary(cse_var_113, vertices_stop_default1, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices1_1_2 = binary(vertices1_1_1, unary(vertices_stop_temp1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			if(unary(any(vertices1_1_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
				break
			priority_vertices1 = get_max_priority(cse_var_111, vertices1_1_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_final_stop1 = binary(vertices_stop_temp1, repeat(unary(priority_vertices1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			polyexp_stop1 = filter_trav_exp_stop(phi_trav_exp1_1_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			polyexp_not_stop1 = filter_trav_exp_not_stop(phi_trav_exp1_1_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			cse_var_101 = polyexp_not_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_98 = (cse_var_101).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_93 = clamp(cse_var_101, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_95 = clamp(cse_var_101, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_89 = clamp(cse_var_98, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_91 = clamp(cse_var_98, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_59 = binary(inner_prod(cse_var_95, (cse_var_117).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_93, (cse_var_115).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_60 = binary(inner_prod((cse_var_91).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_116).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_89).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_114).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_58 = binary(cse_var_59, polyexp_not_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			trav_exp1_4_3 = PolyExpSparse(abs_elem.network, binary(cse_var_60, polyexp_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_58, polyexp_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
			phi_trav_exp1_1_1 = trav_exp1_4_3
		if dummy_mode:
			json_obj = {"num_iterations": while_iteration}
			save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
		cse_var_25 = Llist(abs_elem.network, [1]*(phi_trav_exp1_1_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_102 = phi_trav_exp1_1_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		l_new = binary(binary(inner_prod(clamp(cse_var_102, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_25, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_102, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_25, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp1_1_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		phi_trav_exp2_5_1 = cse_var_44
		while_iteration = -1
		while(True):
			while_iteration += 1
			cse_var_12 = phi_trav_exp2_5_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			vertices2_5_1 = binary(cse_var_12, cse_var_11, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop_default2 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_stop_temp2 = binary(cse_var_113, vertices_stop_default2, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices2_5_2 = binary(vertices2_5_1, unary(vertices_stop_temp2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			if(unary(any(vertices2_5_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
				break
			priority_vertices2 = get_max_priority(cse_var_111, vertices2_5_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_final_stop2 = binary(vertices_stop_temp2, repeat(unary(priority_vertices2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			polyexp_stop2 = filter_trav_exp_stop(phi_trav_exp2_5_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			polyexp_not_stop2 = filter_trav_exp_not_stop(phi_trav_exp2_5_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			cse_var_86 = polyexp_not_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_83 = (cse_var_86).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_78 = clamp(cse_var_86, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_80 = clamp(cse_var_86, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_74 = clamp(cse_var_83, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_76 = clamp(cse_var_83, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_50 = binary(inner_prod(cse_var_80, (cse_var_115).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_78, (cse_var_117).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_51 = binary(inner_prod((cse_var_76).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_114).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_74).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_116).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_49 = binary(cse_var_50, polyexp_not_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			trav_exp2_8_3 = PolyExpSparse(abs_elem.network, binary(cse_var_51, polyexp_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_49, polyexp_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
			phi_trav_exp2_5_1 = trav_exp2_8_3
		if dummy_mode:
			json_obj = {"num_iterations": while_iteration}
			save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
		cse_var_9 = Llist(abs_elem.network, [1]*(phi_trav_exp2_5_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_87 = phi_trav_exp2_5_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		u_new = binary(binary(inner_prod(clamp(cse_var_87, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_9, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_87, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_9, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp2_5_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		return l_new, u_new, cse_var_44, cse_var_44, 
	
	def Relu(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_41 = abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_42 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_46 = binary(cse_var_41, cse_var_42, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		rewrite_new_0 = convert_to_float(cse_var_46)
		cse_var_104 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		l_new = binary(binary(rewrite_new_0, cse_var_41, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_104, rewrite_new_0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_42, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_40 = abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		rewrite_new_1 = convert_to_float(binary(cse_var_40, cse_var_42, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		u_new = binary(binary(rewrite_new_1, cse_var_40, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(binary(cse_var_104, rewrite_new_1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_42, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_38 = prev.convert_to_poly(abs_elem)
		cse_var_47 = repeat(cse_var_38.get_const(), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_48 = repeat(cse_var_38.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_37 = PolyExpSparse(abs_elem.network, 0.0, 0.0)
		cse_var_39 = binary(binary(cse_var_41, cse_var_40, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_42, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_103 = convert_to_float(cse_var_39)
		rewrite_new_2 = repeat((cse_var_103).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_106 = binary(cse_var_104, cse_var_103, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		L_new = PolyExpSparse(abs_elem.network, binary(binary(rewrite_new_2, cse_var_48, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), repeat((binary(cse_var_106, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_37.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), type= type(cse_var_37.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None))).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(binary(cse_var_103, cse_var_47, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(cse_var_106, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_37.get_const(), type= type(cse_var_37.get_const())).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_34 = binary(cse_var_40, cse_var_41, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_36 = binary(cse_var_40, cse_var_34, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_71 = binary(cse_var_36, cse_var_47, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_72 = binary(repeat((cse_var_36).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_48, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_70 = binary(cse_var_71, binary(binary(cse_var_40, cse_var_41, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_34, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_32 = PolyExpSparse(abs_elem.network, 0.0, cse_var_42)
		cse_var_33 = binary(cse_var_40, cse_var_42, operator.lt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_68 = where(cse_var_33, cse_var_32.get_const(), cse_var_70, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_69 = where(repeat((cse_var_33).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_32.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), cse_var_72, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		U_new = PolyExpSparse(abs_elem.network, where(repeat((cse_var_46).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_48, cse_var_69, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , where(cse_var_46, cse_var_47, cse_var_68, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		return l_new, u_new, L_new, U_new, 
	
