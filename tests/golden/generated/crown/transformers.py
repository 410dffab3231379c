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
		cse_var_21 = prev.dot(curr.get_metadata('weight', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), abs_elem.get_poly_size(), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1, mats_input = 'rhs')
		cse_var_20 = repeat(curr.get_metadata('bias', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		cse_var_63 = cse_var_21.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_43 = PolyExpSparse(abs_elem.network, cse_var_63 , binary(cse_var_21.get_const(), cse_var_20, operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
		cse_var_123 = binary(get_dims(cse_var_63, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), 1, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		vertices_stop1 = False
		cse_var_10 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size]))
		cse_var_126 = unary(Llist(abs_elem.network, [1]*(cse_var_123), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist()).get_metadata('layer', batch_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.neg, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_125 = Llist(abs_elem.network, [1]*(cse_var_123), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_127 = abs_elem.get_elem('L', cse_var_125, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_128 = abs_elem.get_elem('U', cse_var_125, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_130 = cse_var_128.get_const()
		cse_var_129 = cse_var_128.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_132 = cse_var_127.get_const()
		cse_var_131 = cse_var_127.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		phi_trav_exp1_1_1 = cse_var_43
		while_iteration = -1
		while(True):
			while_iteration += 1
			cse_var_24 = phi_trav_exp1_1_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			vertices1_1_1 = binary(cse_var_24, cse_var_10, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop_default1 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_stop_temp1 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=vertices_stop1, type= type(vertices_stop1)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size])), vertices_stop_default1, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices1_1_2 = binary(vertices1_1_1, unary(vertices_stop_temp1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			if(unary(any(vertices1_1_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
				break
			priority_vertices1 = get_max_priority(cse_var_126, vertices1_1_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_final_stop1 = binary(vertices_stop_temp1, repeat(unary(priority_vertices1, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			polyexp_stop1 = filter_trav_exp_stop(phi_trav_exp1_1_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			polyexp_not_stop1 = filter_trav_exp_not_stop(phi_trav_exp1_1_1, vertices_final_stop1, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			cse_var_103 = polyexp_not_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_100 = (cse_var_103).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_95 = clamp(cse_var_103, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_97 = clamp(cse_var_103, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_91 = clamp(cse_var_100, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_93 = clamp(cse_var_100, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_55 = binary(inner_prod(cse_var_97, (cse_var_132).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_95, (cse_var_130).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_56 = binary(inner_prod((cse_var_93).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_131).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_91).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_129).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_54 = binary(cse_var_55, polyexp_not_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			trav_exp1_4_3 = PolyExpSparse(abs_elem.network, binary(cse_var_56, polyexp_stop1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_54, polyexp_stop1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
			phi_trav_exp1_1_1 = trav_exp1_4_3
		if dummy_mode:
			json_obj = {"num_iterations": while_iteration}
			save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
		cse_var_22 = Llist(abs_elem.network, [1]*(phi_trav_exp1_1_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_104 = phi_trav_exp1_1_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		l_new = binary(binary(inner_prod(clamp(cse_var_104, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_22, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_104, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_22, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp1_1_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		vertices_stop2 = False
		phi_trav_exp2_5_1 = cse_var_43
		while_iteration = -1
		while(True):
			while_iteration += 1
			cse_var_11 = phi_trav_exp2_5_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			vertices2_5_1 = binary(cse_var_11, cse_var_10, operator.ne, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices_stop_default2 = get_default_stop([batch_size, curr_size, poly_size], abs_elem, batch_size, curr_size, poly_size, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_stop_temp2 = binary(SparseTensor([], [], 0, torch.tensor([]), dense_const=vertices_stop2, type= type(vertices_stop2)).unsqueeze(0).unsqueeze(1).unsqueeze(2).repeat(torch.tensor([batch_size, curr_size, poly_size])), vertices_stop_default2, operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			vertices2_5_2 = binary(vertices2_5_1, unary(vertices_stop_temp2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.and_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			if(unary(any(vertices2_5_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)):
				break
			priority_vertices2 = get_max_priority(cse_var_126, vertices2_5_2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			vertices_final_stop2 = binary(vertices_stop_temp2, repeat(unary(priority_vertices2, operator.not_, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1), torch.tensor([batch_size, curr_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.or_, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			polyexp_stop2 = filter_trav_exp_stop(phi_trav_exp2_5_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			polyexp_not_stop2 = filter_trav_exp_not_stop(phi_trav_exp2_5_1, vertices_final_stop2, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			cse_var_88 = polyexp_not_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			cse_var_85 = (cse_var_88).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_80 = clamp(cse_var_88, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_82 = clamp(cse_var_88, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_76 = clamp(cse_var_85, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_78 = clamp(cse_var_85, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_46 = binary(inner_prod(cse_var_82, (cse_var_130).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_80, (cse_var_132).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_47 = binary(inner_prod((cse_var_78).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_129).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_76).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_131).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			cse_var_45 = binary(cse_var_46, polyexp_not_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
			trav_exp2_8_3 = PolyExpSparse(abs_elem.network, binary(cse_var_47, polyexp_stop2.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(cse_var_45, polyexp_stop2.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
			phi_trav_exp2_5_1 = trav_exp2_8_3
		if dummy_mode:
			json_obj = {"num_iterations": while_iteration}
			save_capture("jit_while/while_iterations_layer_" + str(layer_index) + "_while_" + str(-1) + ".json", json_obj)
		cse_var_8 = Llist(abs_elem.network, [1]*(phi_trav_exp2_5_1.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
		cse_var_89 = phi_trav_exp2_5_1.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		u_new = binary(binary(inner_prod(clamp(cse_var_89, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('u', cse_var_8, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(clamp(cse_var_89, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (abs_elem.get_elem('l', cse_var_8, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), phi_trav_exp2_5_1.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
		return l_new, u_new, cse_var_43, cse_var_43, 
	
	def Relu(self, abs_elem, prev, curr, poly_size, curr_size, prev_size, input_size, batch_size, layer_index = None):
		cse_var_39 = SparseTensor([], [], 0, torch.tensor([]), dense_const=0.0, type= type(0.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
		cse_var_105 = abs_elem.get_elem('l', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		var_19 = any(binary(cse_var_105, cse_var_39, operator.ge, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
		cse_var_34 = abs_elem.get_elem('U', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		cse_var_106 = abs_elem.get_elem('u', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
		if(var_19):
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "then"})
			L_new_1_0 = abs_elem.get_elem('L', prev, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
			return cse_var_105, cse_var_106, L_new_1_0, cse_var_34, 
		else:
			if dummy_mode:
				save_capture("jit_branch/branch_" + str(layer_index) + "_0.json", {"taken": "else"})
			var_18 = any(binary(cse_var_106, cse_var_39, operator.le, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index=layer_index, counter=-1, inside_while=False, while_number=-1)
			if(var_18):
				if dummy_mode:
					save_capture("jit_branch/branch_" + str(layer_index) + "_2.json", {"taken": "then"})
				l_new_3_1 = 0.0
				u_new_3_1 = 0.0
				cse_var_38 = PolyExpSparse(abs_elem.network, 0.0, cse_var_39)
				return l_new_3_1, u_new_3_1, cse_var_38, cse_var_38, 
			else:
				if dummy_mode:
					save_capture("jit_branch/branch_" + str(layer_index) + "_2.json", {"taken": "else"})
				cse_var_37 = binary(binary(cse_var_39, cse_var_105, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_106, operator.gt, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_122 = convert_to_float(cse_var_37)
				cse_var_121 = SparseTensor([], [], 0, torch.tensor([]), dense_const=1.0, type= type(1.0)).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size]))
				cse_var_124 = binary(cse_var_121, cse_var_122, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				l_new_4_2 = binary(binary(cse_var_122, cse_var_39, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(cse_var_124, cse_var_105, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_35 = prev.convert_to_poly(abs_elem)
				cse_var_36 = PolyExpSparse(abs_elem.network, 0.0, 0.0)
				L_new_4_2 = PolyExpSparse(abs_elem.network, binary(repeat((binary(cse_var_122, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_36.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), type= type(cse_var_36.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None))).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(repeat((cse_var_124).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), repeat(cse_var_35.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None), torch.tensor([batch_size, 1, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1) , binary(binary(cse_var_122, SparseTensor([], [], 0, torch.tensor([]), dense_const=cse_var_36.get_const(), type= type(cse_var_36.get_const())).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), binary(cse_var_124, repeat(cse_var_35.get_const(), torch.tensor([batch_size, 1]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
				cse_var_33 = Llist(abs_elem.network, [1]*(cse_var_34.mat.dims-1), None, None,torch.nonzero(abs_elem.d['llist']).flatten().tolist())
				var_13 = abs_elem.get_elem('U', cse_var_33, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				var_14 = abs_elem.get_elem('L', cse_var_33, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_120 = cse_var_34.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_117 = (cse_var_120).unsqueeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_111 = var_14.get_const()
				cse_var_107 = var_14.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_113 = var_13.get_const()
				cse_var_109 = var_13.get_mat(abs_elem, layer_index=layer_index, counter=-1, inside_while=False, while_number=-1, while_iteration=None)
				cse_var_112 = clamp(cse_var_120, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_114 = clamp(cse_var_120, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_108 = clamp(cse_var_117, 0, False, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_110 = clamp(cse_var_117, 0, True, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_67 = binary(inner_prod(cse_var_114, (cse_var_113).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod(cse_var_112, (cse_var_111).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_68 = binary(inner_prod((cse_var_110).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_109).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), inner_prod((cse_var_108).squeeze(3, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), (cse_var_107).squeeze(1, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_66 = binary(cse_var_67, cse_var_34.get_const(), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_25 = binary(cse_var_106, cse_var_105, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_26 = binary(cse_var_106, cse_var_25, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_64 = binary(cse_var_26, cse_var_66, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				cse_var_65 = binary(repeat((cse_var_26).unsqueeze(2, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), torch.tensor([1, 1, poly_size]), layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_68, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1)
				U_new_4_2 = PolyExpSparse(abs_elem.network, cse_var_65 , binary(cse_var_64, binary(binary(binary(cse_var_106, cse_var_105, operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), SparseTensor([], [], 0, torch.tensor([]), dense_const=binary(0.0, 1.0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), type= type(binary(0.0, 1.0, operator.sub, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))).unsqueeze(0).unsqueeze(1).repeat(torch.tensor([batch_size, curr_size])), operator.mul, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), cse_var_25, operator.truediv, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1), operator.add, layer_index = layer_index, counter = -1, inside_while = False, while_number = -1))
				return l_new_4_2, cse_var_106, L_new_4_2, U_new_4_2, 
	
